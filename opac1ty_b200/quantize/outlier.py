"""Outlier-row detection (API of opacc1ty/quantize/outlier.py).

Outliers are whole output rows: the top max(1, int(M * fraction)) rows by L2 norm, plus every row
whose norm exceeds min_magnitude_ratio x the median norm (outlier.py:84-112).  They are kept as
dense fp16 rows and zeroed in the matrix handed to k-means (outlier.py:146-168).

mode="element" keeps single weights instead (the "sparse_outlier" layers the reference's format
reserves): the max(1, int(M * K * fraction)) weights of largest magnitude, as (row, col) fp16
entries; in the matrix handed to k-means each is clipped to the largest magnitude of the other
weights of its row, so the codebooks fit the rest of the row.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch


@dataclass
class OutlierConfig:
    fraction: float = 0.01
    detection_method: str = "magnitude"
    min_magnitude_ratio: float = 5.0
    mode: str = "row"   # "row" (the reference's) or "element"


class OutlierDetector:
    def __init__(self, config: Optional[OutlierConfig] = None):
        self.config = config or OutlierConfig()

    def detect(self, weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(outlier_mask [M] bool, channel_norms [M])."""
        if self.config.detection_method == "magnitude":
            return self._detect_by_magnitude(weight)
        if self.config.detection_method == "sensitivity":
            return self._detect_by_sensitivity(weight)
        raise ValueError(f"Unknown detection method: {self.config.detection_method}")

    def _detect_by_magnitude(self, weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        norms = weight.norm(dim=1)
        M = norms.numel()
        k = max(1, int(M * self.config.fraction))
        top = norms.sort(descending=True).indices[:k]
        mask = torch.zeros(M, dtype=torch.bool, device=weight.device)
        mask[top] = True
        mask |= norms > self.config.min_magnitude_ratio * norms.median()
        return mask, norms

    def _detect_by_sensitivity(self, weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Error of a per-row 4-level uniform quantizer (outlier.py:114-144), all rows at once."""
        norms = weight.norm(dim=1)
        lo = weight.min(dim=1, keepdim=True).values
        hi = weight.max(dim=1, keepdim=True).values
        step = (hi - lo) / 3
        safe = torch.where(step > 0, step, torch.ones_like(step))
        q = torch.round((weight - lo) / safe) * safe + lo
        sens = ((weight - q) ** 2).sum(dim=1)
        sens = torch.where((hi > lo).squeeze(1), sens, torch.zeros_like(sens))
        M = norms.numel()
        k = max(1, int(M * self.config.fraction))
        mask = torch.zeros(M, dtype=torch.bool, device=weight.device)
        mask[sens.sort(descending=True).indices[:k]] = True
        return mask, norms

    def extract_outliers(self, weight: torch.Tensor, outlier_mask: torch.Tensor):
        """(dense weight with outlier rows zeroed, fp16 outlier rows, row ids int64)."""
        dense = weight.clone()
        values = weight[outlier_mask].clone().half()
        ids = torch.where(outlier_mask)[0]
        dense[outlier_mask] = 0
        return dense, values, ids

    def detect_elements(self, weight: torch.Tensor) -> torch.Tensor:
        """[M][K] bool: the max(1, int(M * K * fraction)) weights of largest |w| (none for fraction 0)."""
        mask = torch.zeros_like(weight, dtype=torch.bool)
        if self.config.fraction <= 0:
            return mask
        k = max(1, int(weight.numel() * self.config.fraction))
        top = weight.abs().reshape(-1).topk(k, sorted=False).indices
        mask.view(-1)[top] = True
        return mask

    def extract_element_outliers(self, weight: torch.Tensor, mask: torch.Tensor):
        """(weight with each outlier clipped to its row's largest other magnitude, positions
        [nnz][2] int64 (row, col) in row-major order, fp16 values [nnz])."""
        pos = mask.nonzero()
        values = weight[mask].half()
        rest = torch.where(mask, torch.zeros_like(weight), weight.abs()).amax(dim=1, keepdim=True)
        clipped = torch.maximum(torch.minimum(weight, rest), -rest)
        dense = torch.where(mask, clipped, weight)
        return dense, pos, values

