"""Per-row codebook learning (API of opacc1ty/quantize/codebook.py), vectorised over rows.

Same algorithm as the reference -- k-means++ seeding on each row's sub-vectors
(codebook.py:122-165), Lloyd iterations with empty clusters keeping their centroid and a global
convergence test (codebook.py:167-213), nearest-centroid assignment (codebook.py:215-233) -- but
every step runs on all rows at once (batched multinomial, scatter-add means) instead of Python
loops over rows, and it also runs on CUDA.  Random draws are made in a different order than the
reference's per-row loop, so seeded results are not bit-identical to it; the assignment step is.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch


@dataclass
class CodebookConfig:
    n_bits: int = 2
    sub_vector_size: int = 8
    n_iters: int = 100
    n_samples: int = 65536
    convergence_threshold: float = 1e-5
    use_error_feedback: bool = True


class CodebookLearner:
    ROW_CHUNK = 1024

    def __init__(self, config: Optional[CodebookConfig] = None):
        self.config = config or CodebookConfig()
        self.n_entries = 2 ** self.config.n_bits
        self.svs = self.config.sub_vector_size

    def learn(self, weight: torch.Tensor, device: str = "cpu") -> Tuple[torch.Tensor, torch.Tensor]:
        """(codebooks [M][n_entries][svs] fp16, indices [M][in_features // svs] uint8)."""
        out_f, in_f = weight.shape
        pad = (self.svs - in_f % self.svs) % self.svs
        if pad:
            weight = torch.nn.functional.pad(weight, (0, pad))
        groups = weight.reshape(out_f, -1, self.svs).to(device=device, dtype=torch.float32)
        cb = self._initialize_codebooks(groups)
        cb, idx = self._lloyd_iteration(groups, cb)
        if pad:
            idx = idx[:, : in_f // self.svs]
        return cb.half(), idx.to(torch.uint8)

    def _initialize_codebooks(self, groups: torch.Tensor) -> torch.Tensor:
        M, G, svs = groups.shape
        dev = groups.device
        n_sample = min(self.config.n_samples, G)
        if n_sample < G:
            pick = torch.rand(M, G, device=dev).argsort(dim=1)[:, :n_sample]
            samples = torch.gather(groups, 1, pick.unsqueeze(-1).expand(-1, -1, svs))
        else:
            samples = groups
        rows = torch.arange(M, device=dev)
        cb = torch.zeros(M, self.n_entries, svs, device=dev)
        cb[:, 0] = samples[rows, torch.randint(0, n_sample, (M,), device=dev)]
        min_d = None
        for k in range(1, self.n_entries):
            d = ((samples - cb[:, k - 1 : k]) ** 2).sum(dim=2)  # [M, n_sample]
            min_d = d if min_d is None else torch.minimum(min_d, d)
            total = min_d.sum(dim=1, keepdim=True)
            degenerate = total < 1e-10
            probs = torch.where(degenerate, torch.ones_like(min_d), min_d)
            nxt = torch.multinomial(probs, 1).squeeze(1)
            cb[:, k] = samples[rows, nxt]
        return cb

    def _assign(self, groups: torch.Tensor, codebooks: torch.Tensor) -> torch.Tensor:
        out = torch.empty(groups.shape[:2], dtype=torch.long, device=groups.device)
        for r0 in range(0, groups.shape[0], self.ROW_CHUNK):
            g = groups[r0 : r0 + self.ROW_CHUNK].unsqueeze(2)
            c = codebooks[r0 : r0 + self.ROW_CHUNK].unsqueeze(1)
            out[r0 : r0 + self.ROW_CHUNK] = ((g - c) ** 2).sum(dim=3).argmin(dim=2)
        return out

    def _lloyd_iteration(self, groups: torch.Tensor, codebooks: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        M, G, svs = groups.shape
        E = self.n_entries
        for _ in range(self.config.n_iters):
            idx = self._assign(groups, codebooks)
            sums = torch.zeros(M, E, svs, device=groups.device)
            sums.scatter_add_(1, idx.unsqueeze(-1).expand(-1, -1, svs), groups)
            counts = torch.zeros(M, E, device=groups.device)
            counts.scatter_add_(1, idx, torch.ones_like(idx, dtype=torch.float32))
            new = torch.where(counts.unsqueeze(-1) > 0, sums / counts.clamp(min=1).unsqueeze(-1), codebooks)
            movement = float(((new - codebooks) ** 2).sum())
            if movement < self.config.convergence_threshold:
                break
            codebooks = new
        return codebooks, self._assign(groups, codebooks)
