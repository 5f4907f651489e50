"""Quantization pipeline (API of opacc1ty/quantize/vq.py), vectorised over rows.

Per layer (vq.py:149-200): detect outlier rows and zero them, learn 4-entry per-row codebooks,
optionally re-assign indices with error feedback, and return the reference's layer dict.  Error
feedback (vq.py:202-235) is sequential along K within a row but independent across rows, so it
runs as one vector step per group over all rows; with identical codebooks its indices are the
reference's, element for element (distance sums and argmin ties are the same).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from .codebook import CodebookConfig, CodebookLearner
from .outlier import OutlierConfig, OutlierDetector

VERSION = "1.0.2"  # version string the reference writes into quantize_config (vq.py:144)


@dataclass
class QuantizeConfig:
    bits: int = 2
    sub_vector_size: int = 8
    outlier_fraction: float = 0.01
    use_error_feedback: bool = True
    codebook_iters: int = 100
    group_dim: int = 0
    device: str = "cpu"   # "cpu", "mps" or "cuda"
    outlier_mode: str = "row"   # "row" (whole rows, the reference's) or "element" (single weights, COO)


class VectorQuantizer:
    def __init__(self, config: Optional[QuantizeConfig] = None):
        self.config = config or QuantizeConfig()
        self.codebook_learner = CodebookLearner(CodebookConfig(
            n_bits=self.config.bits, sub_vector_size=self.config.sub_vector_size,
            n_iters=self.config.codebook_iters, use_error_feedback=self.config.use_error_feedback))
        if self.config.outlier_mode not in ("row", "element"):
            raise ValueError(f"outlier_mode must be 'row' or 'element', got {self.config.outlier_mode!r}")
        self.outlier_detector = OutlierDetector(OutlierConfig(fraction=self.config.outlier_fraction,
                                                              mode=self.config.outlier_mode))

    def _device(self) -> torch.device:
        d = self.config.device
        if d == "cuda" and not torch.cuda.is_available():
            raise RuntimeError("QuantizeConfig.device='cuda' but no CUDA device is available")
        return torch.device(d)

    def quantize_model(self, state_dict: Dict[str, torch.Tensor], model_config: dict,
                       progress: bool = True) -> Dict[str, dict]:
        """2-D tensors with both dimensions > 64 are quantized; the rest pass through as fp16
        (vq.py:116-127)."""
        results: Dict[str, dict] = {}
        todo = []
        for name, t in state_dict.items():
            if t.dim() == 2 and t.shape[0] > 64 and t.shape[1] > 64:
                todo.append((name, t))
            else:
                results[name] = {"type": "fp16_passthrough", "shape": tuple(t.shape), "data": t.half(),
                                 "compression_ratio": 1.0}
        it = todo
        if progress:
            try:
                from tqdm import tqdm

                it = tqdm(todo, desc="Quantizing layers")
            except ImportError:
                pass
        for name, w in it:
            r = self.quantize_layer(w.float())
            r["original_name"] = name
            results[name] = r
        results["_model_config"] = model_config
        results["_quantize_config"] = {"bits": self.config.bits, "sub_vector_size": self.config.sub_vector_size,
                                       "outlier_fraction": self.config.outlier_fraction,
                                       "opacc1ty_version": VERSION}
        return results

    def quantize_layer(self, weight: torch.Tensor) -> dict:
        out_f, in_f = weight.shape
        original_bytes = weight.numel() * 2
        dev = self._device()
        weight = weight.to(device=dev, dtype=torch.float32)
        if self.config.outlier_mode == "element":
            return self._quantize_layer_element(weight, original_bytes)
        mask, _ = self.outlier_detector.detect(weight)
        dense, values, ids = self.outlier_detector.extract_outliers(weight, mask)
        cb, idx = self.codebook_learner.learn(dense, device=str(dev))
        if self.config.use_error_feedback:
            cb, idx = self._apply_error_feedback(dense, cb, idx)
        comp = self._compute_compressed_size(out_f, in_f, len(ids), len(cb), cb.shape[1])
        return {
            "type": "quantized",
            "shape": (out_f, in_f),
            "codebooks": cb.cpu().half(),
            "indices": idx.cpu(),
            "outlier_values": values.cpu() if len(ids) > 0 else None,
            "outlier_indices": ids.cpu() if len(ids) > 0 else None,
            "outlier_mask": mask.cpu(),
            "compression_ratio": round(original_bytes / max(comp, 1), 2),
        }

    def _quantize_layer_element(self, weight: torch.Tensor, original_bytes: int) -> dict:
        """Element-wise outliers: a "sparse_outlier" layer (codebooks and indices of the clipped
        matrix, fp16 outlier values at (row, col) positions)."""
        out_f, in_f = weight.shape
        mask = self.outlier_detector.detect_elements(weight)
        dense, pos, values = self.outlier_detector.extract_element_outliers(weight, mask)
        cb, idx = self.codebook_learner.learn(dense, device=str(weight.device))
        if self.config.use_error_feedback:
            cb, idx = self._apply_error_feedback(dense, cb, idx)
        comp = self._compute_compressed_size(out_f, in_f, 0, len(cb), cb.shape[1]) + len(values) * (2 + 8)
        return {
            "type": "sparse_outlier",
            "shape": (out_f, in_f),
            "codebooks": cb.cpu().half(),
            "indices": idx.cpu(),
            "outlier_values": values.cpu(),
            "outlier_indices": pos.cpu(),
            "compression_ratio": round(original_bytes / max(comp, 1), 2),
        }

    def _apply_error_feedback(self, weight: torch.Tensor, codebooks: torch.Tensor,
                              indices: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Carry each group's quantization error into the next group of the same row."""
        M, G = indices.shape
        svs = codebooks.shape[2]
        cb = codebooks.to(weight.device)  # the reference compares against the fp16-rounded table
        err = torch.zeros(M, svs, device=weight.device, dtype=weight.dtype)
        out = indices.clone().to(weight.device)
        rows = torch.arange(M, device=weight.device)
        for g in range(G):
            target = weight[:, g * svs:(g + 1) * svs] + err
            d = ((cb - target.unsqueeze(1)) ** 2).sum(dim=2)
            best = d.argmin(dim=1)
            out[:, g] = best.to(out.dtype)
            err = target - cb[rows, best]
        return codebooks, out.to(indices.device)

    def _compute_compressed_size(self, out_features: int, in_features: int, n_outliers: int, n_groups: int,
                                 n_entries: int) -> int:
        """Byte estimate the reference reports as compression_ratio (vq.py:237-258)."""
        cb = n_groups * n_entries * self.config.sub_vector_size * 2
        idx = n_groups * self.config.sub_vector_size // 4
        return cb + idx + n_outliers * in_features * 2 + n_outliers * 4
