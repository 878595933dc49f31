"""One small, seeded W4A16 case for profilers (ncu): builds the benchmark's
inputs on the GPU and calls the op a few times.

    python -m kernelbench_harbor_b200.profile_case --m 4096 --calls 2
    ncu --set full --clock-control none -k regex:w4a16 -s 1 -c 1 \\
        python -m kernelbench_harbor_b200.profile_case --m 4096 --calls 2

``--moe T`` instead runs the quantised top-2 MoE at the Mixtral shape
(D=4096, H=14336, 8 experts) on T tokens.
"""
from __future__ import annotations

import argparse

import torch


def inputs(M: int, K: int = 14336, N: int = 4096, group: int = 128, seed: int = 1, device: str = "cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    nib = torch.randint(0, 16, (K, N), generator=g, device=device, dtype=torch.int32)
    q = torch.zeros(K, N // 8, dtype=torch.int32, device=device)
    for i in range(8):
        q |= nib[:, i::8] << (4 * i)
    s = (torch.rand(K // group, N, generator=g, device=device) * 0.018 + 0.002).half()
    z = torch.randint(0, 16, (K // group, N), generator=g, device=device).half()
    x = torch.randn(M, K, generator=g, device=device).half()
    return x, q, s, z


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=16)
    ap.add_argument("--calls", type=int, default=2)
    ap.add_argument("--moe", type=int, default=0, help="tokens of a Mixtral-shape MoE call instead")
    args = ap.parse_args()
    from . import ops
    if args.moe:
        from .modules import QuantizedMoE
        T, D, H, E = args.moe, 4096, 14336, 8
        g = torch.Generator(device="cuda").manual_seed(3)
        x = torch.randn(T, D, generator=g, device="cuda").half()
        logits = (x.float() @ (torch.randn(E, D, generator=g, device="cuda") * 0.02).t()).half()
        ws = []
        for (kk, nn) in ((D, H), (D, H), (H, D)):
            parts = [inputs(1, K=kk, N=nn, seed=10 * e + len(ws))[1:] for e in range(E)]
            ws += [torch.stack([p[i] for p in parts]) for i in range(3)]
        mod = QuantizedMoE()
        for _ in range(args.calls):
            mod(x, logits, *ws)
        torch.cuda.synchronize()
        print("ok")
        return
    x, q, s, z = inputs(args.m)
    for _ in range(args.calls):
        ops.w4a16_gemm(x, q, s, z, 128)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
