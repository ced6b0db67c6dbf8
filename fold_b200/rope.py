"""Rotary frequencies of a drafter layer and the cos/sin table the far-query rotation reads.

drafter_rope follows fold/rope.py:14-28 of the reference (neox-style default or Gemma-4
proportional rotary modules only; scaled variants are rejected because FOLD re-rotates queries
with the native frequencies).

rope_table is the device table of the rotation: float32 [rows, rotary_dim] with cos(p f_i) in the
first half and sin(p f_i) in the second, the layout of vLLM's cos_sin_cache. It is formed in
float64 on the host, so the rotation by (D - H) stays exact to float32 at offsets of 1e5 and more
(the reference's kernel forms that angle in float32). Tables are shared by every layer with the
same frequencies on a device.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class Rope:
    inv_freq: torch.Tensor  # [rotary_dim / 2], float32
    rotary_dim: int
    head_dim: int


def drafter_rope(rotary_emb, device=None) -> Rope:
    """Frequencies of a vLLM rotary module (RotaryEmbedding or Gemma4RotaryEmbedding, neox)."""
    name = type(rotary_emb).__name__
    if name not in {"RotaryEmbedding", "Gemma4RotaryEmbedding"}:
        raise ValueError(f"unsupported rotary embedding: {name}")
    if not rotary_emb.is_neox_style:
        raise ValueError("only neox-style rotary embeddings are supported")
    freq = rotary_emb._compute_inv_freq(float(rotary_emb.base)).detach().clone()
    freq = freq.to(device=device or rotary_emb.cos_sin_cache.device, dtype=torch.float32)
    dim = int(rotary_emb.rotary_dim)
    if dim != 2 * freq.numel() or not 0 < dim <= rotary_emb.head_size:
        raise ValueError("rotary and head dimensions disagree")
    return Rope(freq, dim, int(rotary_emb.head_size))


def default_inv_freq(theta: float, rotary_dim: int, device=None) -> torch.Tensor:
    """1 / theta^(2i / rotary_dim) as float32 (vLLM's default RotaryEmbedding)."""
    i = np.arange(0, rotary_dim, 2, dtype=np.float64)
    return torch.from_numpy((1.0 / (theta ** (i / rotary_dim))).astype(np.float32)).to(device)


def table_host(inv_freq, rows: int) -> np.ndarray:
    """cos/sin table [rows, 2 * len(inv_freq)] float32, computed in float64."""
    f = np.asarray(inv_freq.detach().cpu() if isinstance(inv_freq, torch.Tensor) else inv_freq, dtype=np.float64)
    out = np.empty((rows, 2 * f.size), dtype=np.float32)
    step = 1 << 16
    for a in range(0, rows, step):
        ang = np.arange(a, min(rows, a + step), dtype=np.float64)[:, None] * f[None, :]
        out[a:a + ang.shape[0], :f.size] = np.cos(ang)
        out[a:a + ang.shape[0], f.size:] = np.sin(ang)
    return out


_tables: dict = {}
_tables_lock = threading.Lock()


def rope_table(inv_freq: torch.Tensor, rows: int, device) -> torch.Tensor:
    """Shared device table with at least `rows` rows for these frequencies."""
    device = torch.device(device)
    key = (np.asarray(inv_freq.detach().cpu(), dtype=np.float32).tobytes(), str(device))
    with _tables_lock:
        t = _tables.get(key)
        if t is None or t.shape[0] < rows:
            t = torch.from_numpy(table_host(inv_freq, rows)).to(device)
            _tables[key] = t
        return t
