"""Child process of test_explicit_split_gpu.py: computes a fixed set of products on cuda:0 (the
environment decides which split path the library takes) and saves them to the .npz named by
argv[1]."""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import mensurflow_b200 as mf  # noqa: E402


def cases():
    """(name, thunk) pairs; every input comes from a fixed seed, so both processes see the same."""
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(2024)

    def t(*shape, scale=1.0):
        return torch.from_numpy((rng.standard_normal(shape) * scale).astype(np.float32)).to(dev)

    a1, b1, c1 = t(1024, 384), t(384, 512), t(1024, 512)
    a2, b2 = t(700, 256), t(256, 96)
    a3, b3, c3, bias3 = t(1000, 100), t(100, 1000), t(1000, 1000), t(1000, scale=0.1)
    q, k, v = (t(2, 300, 128, scale=1 / np.sqrt(128)) for _ in range(3))
    return [
        ("gemm_smem_split", lambda: mf.gemm(a1, b1, 0.5, c1, 1.0)),
        ("gemm_tmem_split", lambda: mf.matmul(a2, b2)),
        ("gemm_short_k", lambda: mf.gemm(a3, b3, 0.5, c3, 1.0, bias=bias3)),
        ("attention_causal", lambda: mf.attention(q, k, v, causal=True, fused=True)),
        ("attention", lambda: mf.attention(q, k, v, causal=False, fused=True)),
    ]


def run():
    out = {name: f().cpu().numpy() for name, f in cases()}
    assert mf.device_status() == 0
    return out


if __name__ == "__main__":
    np.savez(sys.argv[1], **run())
