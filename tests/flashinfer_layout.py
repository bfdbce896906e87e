"""vLLM FlashInfer paged layouts of the golden cases, for the parity tests.

The golden cases hold each layer as a FlashAttention K plane and V plane,
[num_blocks][block_size][heads][head_bytes] bytes each.  FlashInfer keeps K
and V of a block side by side, [num_blocks][2][...], token-major (NHD) or,
as vLLM does on sm_100, head-major (HND: [num_blocks][2][heads][block_size]
[head_bytes]), and hands the connector a view shaped [num_blocks, 2,
block_size, heads, head_dim].  The same logical KV in either layout must
give the same record bytes.
"""
from __future__ import annotations

import numpy as np
import torch

from tests.golden import gen


def head_bytes_of(case: dict) -> int:
    """bytes of one head of one token: 128 bf16 elements when the unit holds
    whole heads of that size, else the whole unit is one head"""
    unit = gen.unit_of(case)
    return 256 if unit % 256 == 0 else unit


def heads_of(case: dict) -> int:
    return gen.unit_of(case) // head_bytes_of(case)


def to_flashinfer(case: dict, k, v, hnd: bool) -> list[np.ndarray]:
    """per-layer physical bytes of FlashInfer tensors holding planes k, v
    (lists of flat uint8 arrays, one per layer)"""
    nb, bs, H, hb = case["num_blocks"], case["block_size"], heads_of(case), head_bytes_of(case)
    out = []
    for kl, vl in zip(k, v):
        planes = [a.reshape(nb, bs, H, hb) for a in (kl, vl)]
        if hnd:
            planes = [p.transpose(0, 2, 1, 3) for p in planes]
        out.append(np.ascontiguousarray(np.stack(planes, axis=1)).reshape(-1))
    return out


def from_flashinfer(case: dict, layers, hnd: bool):
    """inverse of to_flashinfer: (k planes, v planes) as flat uint8 arrays"""
    nb, bs, H, hb = case["num_blocks"], case["block_size"], heads_of(case), head_bytes_of(case)
    k, v = [], []
    for a in layers:
        x = a.reshape(nb, 2, H, bs, hb) if hnd else a.reshape(nb, 2, bs, H, hb)
        for i, dst in ((0, k), (1, v)):
            p = x[:, i]
            if hnd:
                p = p.transpose(0, 2, 1, 3)
            dst.append(np.ascontiguousarray(p).reshape(-1))
    return k, v


def as_vllm_view(case: dict, phys: torch.Tensor, hnd: bool) -> torch.Tensor:
    """the [num_blocks, 2, block_size, heads, head_dim] view vLLM passes to
    a connector, over flat physical bytes `phys` (element size case['elt'])"""
    nb, bs, H, hb = case["num_blocks"], case["block_size"], heads_of(case), head_bytes_of(case)
    dt = {1: torch.uint8, 2: torch.int16, 4: torch.int32}[case["elt"]]
    d = hb // case["elt"]
    t = phys.view(dt)
    if hnd:
        return t.view(nb, 2, H, bs, d).permute(0, 1, 3, 2, 4)
    return t.view(nb, 2, bs, H, d)


def as_flash_attn_view(case: dict, k_plane: torch.Tensor, v_plane: torch.Tensor) -> torch.Tensor:
    """a [2, num_blocks, block_size, heads, head_dim] tensor (the reference
    layout) with the bytes of two flat planes"""
    nb, bs, H, hb = case["num_blocks"], case["block_size"], heads_of(case), head_bytes_of(case)
    dt = {1: torch.uint8, 2: torch.int16, 4: torch.int32}[case["elt"]]
    return torch.stack([k_plane, v_plane]).view(dt).view(2, nb, bs, H, hb // case["elt"])
