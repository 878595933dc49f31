"""Generate the golden fixtures in this folder from the reference modules.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py --ref <path to kernelbench-harbor checkout>

It imports the reference task modules unmodified (their ``Model`` classes are
device-agnostic; only ``get_inputs`` hard-codes CUDA, so the inputs are rebuilt
here on the CPU with the same recipe and a seeded generator), evaluates them on
the CPU, and writes one ``.npz`` per case with the inputs, the module's output in
the activation dtype (``y_module``) and the grader's fp32 ground truth
(``y_fp32``, floating inputs upcast, integer inputs unchanged -- the convention
of ``common/kb_verifier.py:194-196``).  bf16 tensors are stored as uint16 bit
patterns.  The fixtures are committed; the GPU box never needs the reference.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (tag, task dir under tasks/quant_w4a16_pa, M, K, N, group, dtype, scale distribution)
W4A16_CASES = [
    ("w4a16_m16_k256_n128_g128_fp16", "quant_w4a16_pa__llama3_8b_down__g128__fp16", 16, 256, 128, 128, "fp16", "bj"),
    ("w4a16_m5_k512_n256_g128_fp16", "quant_w4a16_pa__llama3_8b_down__g128__fp16", 5, 512, 256, 128, "fp16", "ref"),
    ("w4a16_m1_k384_n64_g128_fp16", "quant_w4a16_pa__llama3_8b_gate__g128__fp16", 1, 384, 64, 128, "fp16", "bj"),
    ("w4a16_m17_k256_n96_g128_fp16", "quant_w4a16_pa__qwen2_7b_down__g128__fp16", 17, 256, 96, 128, "fp16", "bj"),
    ("w4a16_m16_k256_n128_g64_fp16", "quant_w4a16_pa__llama3_8b_down__g64__fp16", 16, 256, 128, 64, "fp16", "bj"),
    ("w4a16_m16_k256_n128_g128_bf16", "quant_w4a16_pa__llama3_8b_down__g128__bf16", 16, 256, 128, 128, "bf16", "bj"),
    ("w4a16_m130_k256_n256_g128_fp16", "quant_w4a16_pa__llama3_8b_down__g128__fp16", 130, 256, 256, 128, "fp16", "bj"),
]


def load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def tdt(dtype: str):
    return {"fp16": torch.float16, "bf16": torch.bfloat16}[dtype]


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def w4a16_inputs(M, K, N, group, dtype, dist, seed):
    """get_inputs of QUANT_REF (generate_tasks.py:63-73) on the CPU, seeded.  With
    dist == "bj" the scales follow the benchmark's U[0.002, 0.02] instead of the
    reference's randn*0.01; everything else is the reference recipe."""
    g = torch.Generator().manual_seed(seed)
    nib = torch.randint(0, 16, (K, N), generator=g, dtype=torch.int64)
    packed = torch.zeros(K, N // 8, dtype=torch.int64)
    for i in range(8):
        packed |= nib[:, i::8] << (4 * i)
    qweight = packed.to(torch.int32)
    x = torch.randn(M, K, generator=g).to(tdt(dtype))
    if dist == "bj":
        scales = (torch.rand(K // group, N, generator=g) * 0.018 + 0.002).to(tdt(dtype))
    else:
        scales = (torch.randn(K // group, N, generator=g) * 0.01).to(tdt(dtype))
    zeros = torch.randint(0, 16, (K // group, N), generator=g).to(tdt(dtype))
    return nib, [x, qweight, scales, zeros]


def gt_call(model, inputs):
    gt_inputs = [t.float() if t.is_floating_point() else t for t in inputs]
    return model(*gt_inputs).float()


def make_w4a16(ref_root: str, out: dict):
    for i, (tag, task, M, K, N, group, dtype, dist) in enumerate(W4A16_CASES):
        path = os.path.join(ref_root, "tasks", "quant_w4a16_pa", task, "environment", "reference.py")
        mod = load_module(path, f"ref_{tag}")
        assert mod.GROUP == group, (task, mod.GROUP, group)
        nib, inputs = w4a16_inputs(M, K, N, group, dtype, dist, seed=1000 + i)
        model = mod.Model()
        with torch.no_grad():
            y = model(*inputs)
            y32 = gt_call(model, inputs)
            # identity activations read the module's dequantised weight back exactly
            w_deq = model(torch.eye(K, dtype=tdt(dtype)), *inputs[1:])
        x, qweight, scales, zeros = inputs
        np.savez_compressed(
            os.path.join(HERE, tag + ".npz"),
            nib=nib.numpy().astype(np.uint8), x=to_np(x), qweight=qweight.numpy(),
            scales=to_np(scales), zeros=to_np(zeros), y_module=to_np(y), y_fp32=y32.numpy(), w_dequant=to_np(w_deq),
            meta=json.dumps({"M": M, "K": K, "N": N, "group": group, "dtype": dtype,
                             "dist": dist, "task": task, "seed": 1000 + i}))
        out[tag] = {"M": M, "K": K, "N": N, "group": group, "dtype": dtype, "task": task}


def make_unpack_kat(ref_root: str, out: dict):
    """Known-answer words through the reference unpack: sign bit set, all ones,
    ascending nibbles, and a random column of words."""
    path = os.path.join(ref_root, "tasks", "quant_w4a16_pa",
                        "quant_w4a16_pa__llama3_8b_down__g128__fp16", "environment", "reference.py")
    mod = load_module(path, "ref_unpack")
    words = np.array([0x00000000, 0x80000000, 0xFFFFFFFF, 0x76543210, 0x01234567,
                      0xFEDCBA98, 0x7FFFFFFF, 0x0000000F, 0xF0000000, 0x89ABCDEF,
                      0x12345678, 0xCAFEBABE, 0xDEADBEEF, 0x55555555, 0xAAAAAAAA, 0x0F0F0F0F],
                     dtype=np.uint64).astype(np.uint32).view(np.int32)
    K = 128
    q = np.zeros((K, 16), dtype=np.int32)
    q[0, :] = words
    g = torch.Generator().manual_seed(7)
    q[1:, :] = torch.randint(-2**31, 2**31 - 1, (K - 1, 16), generator=g, dtype=torch.int64).numpy().astype(np.int32)
    qweight = torch.from_numpy(q)
    # scales = 1, zeros = 0 makes the module output x @ nib, so the nibbles read back exactly
    N = 128
    scales = torch.ones(1, N, dtype=torch.float32)
    zeros = torch.zeros(1, N, dtype=torch.float32)
    eye = torch.eye(K, dtype=torch.float32)
    with torch.no_grad():
        nib = mod.Model()(eye, qweight, scales, zeros)
    np.savez_compressed(os.path.join(HERE, "unpack_kat.npz"), qweight=q,
                        nib=nib.numpy().astype(np.uint8))
    out["unpack_kat"] = {"K": K, "N": N}


def make_w8a8(ref_root: str, out: dict):
    path = os.path.join(ref_root, "tasks", "w8a8_smoothquant",
                        "w8a8_smoothquant__llama3_8b_down__M16", "environment", "reference.py")
    mod = load_module(path, "ref_w8a8")
    for i, (M, K, N) in enumerate([(16, 256, 128), (33, 512, 64)]):
        g = torch.Generator().manual_seed(2000 + i)
        x_int8 = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        w_int8 = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int8)
        x_scale = (torch.rand(M, 1, generator=g) * 0.01 + 0.001).to(torch.float16)
        w_scale = (torch.rand(1, N, generator=g) * 0.01 + 0.001).to(torch.float16)
        inputs = [x_int8, w_int8, x_scale, w_scale]
        with torch.no_grad():
            y = mod.Model()(*inputs)
            y32 = gt_call(mod.Model(), inputs)
        tag = f"w8a8_m{M}_k{K}_n{N}"
        np.savez_compressed(os.path.join(HERE, tag + ".npz"), x_int8=x_int8.numpy(),
                            w_int8=w_int8.numpy(), x_scale=x_scale.numpy(), w_scale=w_scale.numpy(),
                            y_module=y.numpy(), y_fp32=y32.numpy())
        out[tag] = {"M": M, "K": K, "N": N}


def make_routing(ref_root: str, out: dict):
    """Top-2 routing of MOE_REF / FUSED_QMOE_REF (generate_tasks.py:171-173,
    368-371), including rows with tied logits, and one small full FUSED_QMOE
    forward for the combine order."""
    path = os.path.join(ref_root, "tasks", "fused_qmoe", "fused_qmoe__mixtral__fp16",
                        "environment", "reference.py")
    mod = load_module(path, "ref_qmoe")
    g = torch.Generator().manual_seed(3000)
    T, E = 256, 8
    logits = torch.randn(T, E, generator=g).to(torch.float16)
    logits[0] = 0.5                       # all equal
    logits[1, :] = torch.tensor([1, 2, 2, 0, -1, 2, 0, 1], dtype=torch.float16)  # three-way tie for 1st
    logits[2, :] = torch.tensor([3, 1, 1, 0, 0, 0, 0, 1], dtype=torch.float16)   # tie for 2nd
    logits[3, :] = torch.tensor([-65504, 0, 0, 0, 0, 0, 0, 65504], dtype=torch.float16)
    probs = torch.softmax(logits.float(), dim=-1)
    topv, topi = probs.topk(2, dim=-1)
    gates = (topv / topv.sum(dim=-1, keepdim=True)).to(torch.float16)
    # small full forward of the reference quantised MoE
    Tm, D, N = 16, 256, 64
    x = torch.randn(Tm, D, generator=g).to(torch.float16)
    qweight = torch.randint(-8, 8, (E, D, N), generator=g, dtype=torch.int8)
    scales = (torch.randn(E, D // 128, N, generator=g) * 0.01).to(torch.float16)
    rl = torch.randn(Tm, E, generator=g).to(torch.float16)
    with torch.no_grad():
        y = mod.Model()(x, qweight, scales, rl)
        y32 = gt_call(mod.Model(), [x, qweight, scales, rl])
    np.savez_compressed(os.path.join(HERE, "moe_routing.npz"), logits=logits.numpy(),
                        topi=topi.numpy().astype(np.int32), gates=gates.numpy(),
                        qmoe_x=x.numpy(), qmoe_qweight=qweight.numpy(), qmoe_scales=scales.numpy(),
                        qmoe_logits=rl.numpy(), qmoe_y_module=y.numpy(), qmoe_y_fp32=y32.numpy())
    out["moe_routing"] = {"T": T, "E": E, "qmoe": [Tm, D, N]}


def make_fp8(ref_root: str, out: dict):
    """FP8_REF (generate_tasks.py:218-237), block 32, for the e4m3 decode table
    and the block-scale broadcast."""
    path = os.path.join(ref_root, "tasks", "fp8_microscale",
                        "fp8_microscale__llama3_8b_down__b32__fp16", "environment", "reference.py")
    mod = load_module(path, "ref_fp8")
    g = torch.Generator().manual_seed(4000)
    M, K, N, B = 16, 256, 64, mod.BLOCK
    x = torch.randn(M, K, generator=g).to(torch.float16)
    w_fp8 = (torch.randn(K, N, generator=g) * 0.3).to(torch.float8_e4m3fn)
    scales = (torch.rand(K // B, N, generator=g) * 0.05 + 0.05).to(torch.float16)
    with torch.no_grad():
        y = mod.Model()(x, w_fp8, scales)
        y32 = gt_call(mod.Model(), [x, w_fp8, scales])
    all_codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    np.savez_compressed(os.path.join(HERE, "fp8_block32.npz"), x=x.numpy(),
                        w_fp8=w_fp8.view(torch.uint8).numpy(), scales=scales.numpy(),
                        y_module=y.numpy(), y_fp32=y32.numpy(), e4m3_table=all_codes.numpy())
    out["fp8_block32"] = {"M": M, "K": K, "N": N, "block": B}


def make_silu_fp8(ref_root: str, out: dict):
    """FUSED_SILU_REF (generate_tasks.py:321-348): SiLU * mul + per-128 dynamic
    e4m3 quantisation, evaluated by the reference module on the CPU."""
    path = os.path.join(ref_root, "tasks", "fused_silu_fp8", "fused_silu_fp8__deepseek_moe__T256__fp16",
                        "environment", "reference.py")
    mod = load_module(path, "ref_silu_fp8")
    g = torch.Generator().manual_seed(5000)
    for dtype in ("fp16", "bf16"):
        T, H = 8, 384
        y = torch.randn(T, 2 * H, generator=g).to(tdt(dtype))
        y[0, :H] = 0.0  # an all-zero group: the scale floor
        y[1, H:H + 128] *= 40.0  # a group whose products are large
        with torch.no_grad():
            o = mod.Model()(y)
        tag = f"silu_fp8_t{T}_h{H}_{dtype}"
        np.savez_compressed(os.path.join(HERE, tag + ".npz"), y=to_np(y), out=o.numpy())
        out[tag] = {"T": T, "H": H, "dtype": dtype, "group": mod.GROUP}


def make_lora(ref_root: str, out: dict):
    """LORA_REF (generate_tasks.py:397-424): int4 base + per-token gathered LoRA."""
    path = os.path.join(ref_root, "tasks", "multi_lora_qgemm", "multi_lora_qgemm__llama3_8b_r16__fp16",
                        "environment", "reference.py")
    mod = load_module(path, "ref_lora")
    g = torch.Generator().manual_seed(6000)
    T, D, N, r, L = 16, 256, 128, 16, 4
    x = torch.randn(T, D, generator=g).to(torch.float16)
    qweight = torch.randint(-8, 8, (D, N), generator=g, dtype=torch.int8)
    scales = (torch.randn(D // 128, N, generator=g) * 0.01).to(torch.float16)
    A = (torch.randn(L, D, r, generator=g) * 0.02).to(torch.float16)
    B = (torch.randn(L, r, N, generator=g) * 0.02).to(torch.float16)
    ids = torch.randint(0, L, (T,), generator=g)
    inputs = [x, qweight, scales, A, B, ids]
    with torch.no_grad():
        y = mod.Model()(*inputs)
        y32 = gt_call(mod.Model(), inputs)
    np.savez_compressed(os.path.join(HERE, "lora_t16_d256_n128_r16.npz"), x=x.numpy(), qweight=qweight.numpy(),
                        scales=scales.numpy(), A=A.numpy(), B=B.numpy(), lora_ids=ids.numpy(),
                        y_module=y.numpy(), y_fp32=y32.numpy())
    out["lora_t16_d256_n128_r16"] = {"T": T, "D": D, "N": N, "r": r, "L": L}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="kernelbench-harbor checkout")
    args = ap.parse_args()
    torch.manual_seed(0)
    out: dict = {}
    make_w4a16(args.ref, out)
    make_unpack_kat(args.ref, out)
    make_w8a8(args.ref, out)
    make_routing(args.ref, out)
    make_fp8(args.ref, out)
    make_silu_fp8(args.ref, out)
    make_lora(args.ref, out)
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump({"torch": torch.__version__, "cases": out}, f, indent=1, sort_keys=True)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    sys.exit(main())
