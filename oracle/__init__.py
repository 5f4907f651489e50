"""CPU oracle package (test infrastructure only; never imported by opac1ty_b200)."""
