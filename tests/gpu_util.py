"""GPU-side helpers for the -m gpu tests: numpy <-> torch CUDA transfer and a
thin driver of the C ABI through lisa_attn.AttnRunner."""
from __future__ import annotations

import numpy as np
import torch

import lisa_attn


def dev_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def dev_inputs(q, k, v, dtype=torch.float32):
    conv = (lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype).contiguous())
    return conv(q), conv(k), conv(v)


def weights(qn, kn) -> lisa_attn.AttentionWeights:
    return lisa_attn.AttentionWeights(dev_bf16(qn), dev_bf16(kn))


def load_cache(runner: lisa_attn.AttnRunner, layer: int, kc: np.ndarray, vc: np.ndarray) -> None:
    k, v = runner.kv_cache(layer)
    k.copy_(dev_bf16(kc).view(k.shape))
    v.copy_(dev_bf16(vc).view(v.shape))
    torch.cuda.synchronize()


def read_cache(runner: lisa_attn.AttnRunner, layer: int):
    k, v = runner.kv_cache(layer)
    torch.cuda.synchronize()
    return to_bits(k), to_bits(v)
