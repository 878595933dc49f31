"""torch custom ops over the C ABI (include/b200q.h).

Each op validates its tensors the way the reference operator would see them
(shapes of QUANT_REF.forward, generate_tasks.py:54-61), makes them contiguous
(as the reference Triton oracle does, common/oracles/quant_w4a16_pa.py:74-77),
allocates the output (callee-allocated, like the oracle's torch.empty at :79)
and calls the library on the current CUDA stream.  No CPU path exists: a CPU
tensor is an error."""
from __future__ import annotations

import threading
from typing import Optional

import torch

from . import _lib

_ws_lock = threading.Lock()
_ws: dict = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch owned by this process, one per (device, stream).
    Kernels return it to the zero state, so it is allocated (and zeroed) once
    and reused; it is never shared by two streams, whose launches could overlap."""
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
            _ws[key] = buf
        return buf


def reset_workspaces() -> None:
    with _ws_lock:
        _ws.clear()


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return _lib.DTYPE_FP16
    if dt == torch.bfloat16:
        return _lib.DTYPE_BF16
    raise TypeError(f"activations must be float16 or bfloat16, got {dt}")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@torch.library.custom_op("b200q::w4a16_gemm", mutates_args=())
def w4a16_gemm(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
               group: int) -> torch.Tensor:
    """y[M, N] = x[M, K] . ((unpack(qweight) - zeros) * scales), y in x.dtype."""
    if not x.is_cuda:
        raise RuntimeError("b200q::w4a16_gemm runs on CUDA tensors only (no CPU implementation)")
    if x.dim() != 2 or qweight.dim() != 2:
        raise ValueError("x must be [M, K] and qweight [K, N/8]")
    if qweight.dtype != torch.int32:
        raise TypeError("qweight must be int32")
    M, K = x.shape
    if qweight.shape[0] != K:
        raise ValueError(f"qweight has {qweight.shape[0]} rows, x has K={K}")
    N = qweight.shape[1] * 8
    if group <= 0 or K % group:
        raise ValueError(f"K={K} is not a multiple of group={group}")
    for name, t in (("scales", scales), ("zeros", zeros)):
        if tuple(t.shape) != (K // group, N):
            raise ValueError(f"{name} must be [{K // group}, {N}], got {tuple(t.shape)}")
    dt = _dtype_code(x.dtype)
    scales = scales.to(x.dtype)
    zeros = zeros.to(x.dtype)
    x, qweight, scales, zeros = (_aligned(t) for t in (x, qweight, scales, zeros))
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0:
        return y
    L = _lib.lib()
    nbytes = L.b200q_w4a16_workspace_bytes(M, N, K, group, x.device.index)
    ws = workspace(x.device, nbytes)
    _lib.check(L.b200q_w4a16_gemm(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                  y.data_ptr(), M, N, K, group, dt, ws.data_ptr(), ws.numel(),
                                  _stream_ptr(x.device)))
    return y


@w4a16_gemm.register_fake
def _(x, qweight, scales, zeros, group):
    return x.new_empty((x.shape[0], qweight.shape[1] * 8))


def _ptr_array(ptrs) -> "ctypes.Array":
    import ctypes
    return (ctypes.c_void_p * len(ptrs))(*[int(p) for p in ptrs])


def w4a16_gemm_peers(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                     group: int, y_ptrs, ldy: int, col0: int, pad_ptrs=None, rank: int = 0) -> None:
    """Columns [col0, col0 + N) of y = x . W from this rank's shard, stored
    into every buffer of ``y_ptrs`` (device addresses of [M, ldy] arrays in
    x.dtype, peers' included).  With ``pad_ptrs`` (every rank's signal pad)
    the kernel orders itself against the peers; without, the caller does
    (``peer_barrier`` before and after)."""
    if not x.is_cuda:
        raise RuntimeError("w4a16_gemm_peers runs on CUDA tensors only (no CPU implementation)")
    M, K = x.shape
    N = qweight.shape[1] * 8
    if qweight.dtype != torch.int32 or qweight.shape[0] != K:
        raise ValueError("qweight must be int32 [K, N/8]")
    dt = _dtype_code(x.dtype)
    scales = scales.to(x.dtype)
    zeros = zeros.to(x.dtype)
    x, qweight, scales, zeros = (_aligned(t) for t in (x, qweight, scales, zeros))
    if M == 0:
        return
    L = _lib.lib()
    ws = workspace(x.device, L.b200q_w4a16_workspace_bytes(M, N, K, group, x.device.index))
    arr = _ptr_array(y_ptrs)
    pads = _ptr_array(pad_ptrs) if pad_ptrs is not None else None
    _lib.check(L.b200q_w4a16_gemm_peers(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                        arr, len(y_ptrs), ldy, col0, pads, rank, M, N, K, group, dt,
                                        ws.data_ptr(), ws.numel(), _stream_ptr(x.device)))


def peer_barrier(pad_ptrs, rank: int, device: torch.device) -> None:
    """Barrier of the len(pad_ptrs) ranks on the current stream (signal pads
    of 64 zeroed uint32 words, every rank's mapped into this process)."""
    L = _lib.lib()
    ws = workspace(device, 256)
    _lib.check(L.b200q_peer_barrier(_ptr_array(pad_ptrs), len(pad_ptrs), rank, ws.data_ptr(),
                                    _stream_ptr(device)))


@torch.library.custom_op("b200q::w8a8_gemm", mutates_args=())
def w8a8_gemm(x_int8: torch.Tensor, w_int8: torch.Tensor, x_scale: torch.Tensor,
              w_scale: torch.Tensor) -> torch.Tensor:
    """y[M, N] = fp16((x_int8 . w_int8) * x_scale * w_scale) (W8A8_REF.forward,
    generate_tasks.py:204-206); x_scale [M, 1] or [M], w_scale [1, N] or [N]."""
    if not x_int8.is_cuda:
        raise RuntimeError("b200q::w8a8_gemm runs on CUDA tensors only (no CPU implementation)")
    if x_int8.dtype != torch.int8 or w_int8.dtype != torch.int8:
        raise TypeError("x_int8 and w_int8 must be int8")
    M, K = x_int8.shape
    if w_int8.shape[0] != K:
        raise ValueError(f"w_int8 has {w_int8.shape[0]} rows, x has K={K}")
    N = w_int8.shape[1]
    xs = x_scale.reshape(-1).to(torch.float16)
    wsc = w_scale.reshape(-1).to(torch.float16)
    if xs.numel() != M or wsc.numel() != N:
        raise ValueError("x_scale must have M entries and w_scale N entries")
    x_int8, w_int8, xs, wsc = (_aligned(t) for t in (x_int8, w_int8, xs, wsc))
    y = torch.empty((M, N), dtype=torch.float16, device=x_int8.device)
    if M == 0:
        return y
    L = _lib.lib()
    ws = workspace(x_int8.device, L.b200q_w8a8_workspace_bytes(M, N, K, x_int8.device.index))
    _lib.check(L.b200q_w8a8_gemm(x_int8.data_ptr(), w_int8.data_ptr(), xs.data_ptr(), wsc.data_ptr(),
                                 y.data_ptr(), M, N, K, ws.data_ptr(), ws.numel(), _stream_ptr(x_int8.device)))
    return y


@w8a8_gemm.register_fake
def _(x_int8, w_int8, x_scale, w_scale):
    return x_int8.new_empty((x_int8.shape[0], w_int8.shape[1]), dtype=torch.float16)


@torch.library.custom_op("b200q::mxfp8_gemm", mutates_args=())
def mxfp8_gemm(a: torch.Tensor, scales_a: torch.Tensor, b: torch.Tensor, scales_b: torch.Tensor) -> torch.Tensor:
    """y[M, N] = fp16(A_deq . B_deq^T) for OCP-MX e4m3 operands (codes as uint8 or
    float8_e4m3fn [M, K] / [N, K], E8M0 scales uint8 [M, K/32] / [N, K/32])."""
    if not a.is_cuda:
        raise RuntimeError("b200q mxfp8_gemm runs on CUDA tensors only")
    a, b = (t.view(torch.uint8) if t.dtype != torch.uint8 else t for t in (a, b))
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K or scales_a.shape != (M, K // 32) or scales_b.shape != (N, K // 32):
        raise ValueError("mxfp8_gemm: shapes must be A [M,K], B [N,K], scales [*, K/32]")
    a, b, scales_a, scales_b = (_aligned(t) for t in (a, b, scales_a, scales_b))
    y = torch.empty((M, N), dtype=torch.float16, device=a.device)
    if M == 0:
        return y
    L = _lib.lib()
    ws = workspace(a.device, L.b200q_mxfp8_workspace_bytes(M, N, K, a.device.index))
    _lib.check(L.b200q_mxfp8_gemm(a.data_ptr(), scales_a.data_ptr(), b.data_ptr(), scales_b.data_ptr(),
                                  y.data_ptr(), M, N, K, ws.data_ptr(), ws.numel(), _stream_ptr(a.device)))
    return y


@mxfp8_gemm.register_fake
def _(a, scales_a, b, scales_b):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.float16)


def mxfp8_gemm_peers(a: torch.Tensor, scales_a: torch.Tensor, b: torch.Tensor, scales_b: torch.Tensor,
                     y_ptrs, ldy: int, col0: int, pad_ptrs=None, rank: int = 0) -> None:
    """Columns [col0, col0 + N) of y = A . B^T from this rank's B shard [N, K],
    stored into every buffer of ``y_ptrs`` ([M, ldy] fp16, peers' included),
    ordered against the peers through ``pad_ptrs`` as in w4a16_gemm_peers."""
    if not a.is_cuda:
        raise RuntimeError("mxfp8_gemm_peers runs on CUDA tensors only (no CPU implementation)")
    a, b = (t.view(torch.uint8) if t.dtype != torch.uint8 else t for t in (a, b))
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K or scales_a.shape != (M, K // 32) or scales_b.shape != (N, K // 32):
        raise ValueError("mxfp8_gemm_peers: shapes must be A [M,K], B [N,K], scales [*, K/32]")
    a, b, scales_a, scales_b = (_aligned(t) for t in (a, b, scales_a, scales_b))
    if M == 0:
        return
    L = _lib.lib()
    ws = workspace(a.device, L.b200q_mxfp8_workspace_bytes(M, N, K, a.device.index))
    pads = _ptr_array(pad_ptrs) if pad_ptrs is not None else None
    _lib.check(L.b200q_mxfp8_gemm_peers(a.data_ptr(), scales_a.data_ptr(), b.data_ptr(), scales_b.data_ptr(),
                                        _ptr_array(y_ptrs), len(y_ptrs), ldy, col0, pads, rank, M, N, K,
                                        ws.data_ptr(), ws.numel(), _stream_ptr(a.device)))


@torch.library.custom_op("b200q::moe_route", mutates_args=())
def moe_route(router_logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                     torch.Tensor]:
    """Top-2 routing + expert-grouped permutation (see include/b200q.h).
    Returns topi [T,2] int32, gates [T,2] (logits dtype), offsets [E+1] int32,
    slot_token [2T] int32, token_slot [T,2] int32."""
    if not router_logits.is_cuda:
        raise RuntimeError("b200q moe_route runs on CUDA tensors only")
    lg = _aligned(router_logits)
    T, E = lg.shape
    dev = lg.device
    topi = torch.empty((T, 2), dtype=torch.int32, device=dev)
    gates = torch.empty((T, 2), dtype=lg.dtype, device=dev)
    offsets = torch.empty((E + 1,), dtype=torch.int32, device=dev)
    slot_token = torch.empty((2 * T,), dtype=torch.int32, device=dev)
    token_slot = torch.empty((T, 2), dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().b200q_moe_route(lg.data_ptr(), T, E, _dtype_code(lg.dtype), topi.data_ptr(),
                                          gates.data_ptr(), offsets.data_ptr(), slot_token.data_ptr(),
                                          token_slot.data_ptr(), _stream_ptr(dev)))
    return topi, gates, offsets, slot_token, token_slot


@moe_route.register_fake
def _(router_logits):
    T, E = router_logits.shape
    i32 = dict(dtype=torch.int32)
    return (router_logits.new_empty((T, 2), **i32), router_logits.new_empty((T, 2)),
            router_logits.new_empty((E + 1,), **i32), router_logits.new_empty((2 * T,), **i32),
            router_logits.new_empty((T, 2), **i32))


def moe_grouped_gemm(x: torch.Tensor, offsets: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                     zeros: torch.Tensor, group: int, up=None) -> torch.Tensor:
    """See moe_grouped_gemm_op; ``up`` = (qweight_up, scales_up, zeros_up) or None."""
    u = up if up is not None else (None, None, None)
    return moe_grouped_gemm_op(x, offsets, qweight, scales, zeros, group, u[0], u[1], u[2])


@torch.library.custom_op("b200q::moe_grouped_gemm", mutates_args=())
def moe_grouped_gemm_op(x: torch.Tensor, offsets: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                        zeros: torch.Tensor, group: int, qweight_up: Optional[torch.Tensor] = None,
                        scales_up: Optional[torch.Tensor] = None,
                        zeros_up: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One launch over all experts.  x [rows, K] grouped by expert (rows of
    expert e at [offsets[e], offsets[e+1]), offsets on the device); qweight
    [E, K, N/8], scales / zeros [E, K/group, N].  Returns y [rows, N] =
    x . W_e, or with ``up = (qweight_up, scales_up, zeros_up)`` the fused
    SiLU(x . Wg_e) * (x . Wu_e)."""
    up = None if qweight_up is None else (qweight_up, scales_up, zeros_up)
    if not x.is_cuda:
        raise RuntimeError("b200q moe_grouped_gemm runs on CUDA tensors only")
    rows, K = x.shape
    E = qweight.shape[0]
    if qweight.dim() != 3 or qweight.shape[1] != K or qweight.dtype != torch.int32:
        raise ValueError("qweight must be int32 [E, K, N/8]")
    N = qweight.shape[2] * 8
    if offsets.dtype != torch.int32 or offsets.numel() != E + 1:
        raise ValueError("offsets must be int32 [E + 1]")
    dt = _dtype_code(x.dtype)
    ts = [_aligned(t) for t in (x, qweight, scales.to(x.dtype), zeros.to(x.dtype), offsets)]
    if up is not None:
        ts += [_aligned(up[0]), _aligned(up[1].to(x.dtype)), _aligned(up[2].to(x.dtype))]
        if tuple(ts[5].shape) != tuple(qweight.shape):
            raise ValueError("up-projection qweight must match the gate's shape")
    y = torch.empty((rows, N), dtype=x.dtype, device=x.device)
    if rows == 0:
        return y
    ws = workspace(x.device, 256)
    ptr = lambda i: ts[i].data_ptr() if i < len(ts) else None  # noqa: E731
    _lib.check(_lib.lib().b200q_moe_grouped_gemm(ptr(0), ptr(1), ptr(2), ptr(3), ptr(5), ptr(6), ptr(7), ptr(4), E,
                                                 y.data_ptr(), rows, N, K, group, dt, ws.data_ptr(), ws.numel(),
                                                 _stream_ptr(x.device)))
    return y


@moe_grouped_gemm_op.register_fake
def _(x, offsets, qweight, scales, zeros, group, qweight_up=None, scales_up=None, zeros_up=None):
    return x.new_empty((x.shape[0], qweight.shape[2] * 8))


def ep_pack(x: torch.Tensor, offsets: torch.Tensor, slot_token: torch.Tensor, token_slot: torch.Tensor,
            n_experts: int, world: int, capacity: int):
    """Send buffer [world * capacity, D + 8] of an expert-parallel exchange
    (see include/b200q.h) and pair_slot [T, 2] int32."""
    T, D = x.shape
    x = _aligned(x)
    send = torch.empty((world * capacity, D + 8), dtype=x.dtype, device=x.device)
    pair_slot = torch.empty((T, 2), dtype=torch.int32, device=x.device)
    _lib.check(_lib.lib().b200q_ep_pack(x.data_ptr(), T, D, _dtype_code(x.dtype), offsets.data_ptr(),
                                        slot_token.data_ptr(), token_slot.data_ptr(), n_experts, world, capacity,
                                        send.data_ptr(), pair_slot.data_ptr(), _stream_ptr(x.device)))
    return send, pair_slot


def ep_regroup(recv: torch.Tensor, n_local: int):
    """(loc_offsets [n_local + 1], src [R], row_pos [R]) int32 for received rows [R, D + 8]."""
    R, D8 = recv.shape
    dev = recv.device
    loc = torch.empty(n_local + 1, dtype=torch.int32, device=dev)
    src = torch.empty(R, dtype=torch.int32, device=dev)
    pos = torch.empty(R, dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().b200q_ep_regroup(recv.data_ptr(), R, D8 - 8, _dtype_code(recv.dtype), n_local,
                                           loc.data_ptr(), src.data_ptr(), pos.data_ptr(), _stream_ptr(dev)))
    return loc, src, pos


def ep_gather(src: torch.Tensor, idx: torch.Tensor, D: int, out: torch.Tensor) -> torch.Tensor:
    """out[j, :D] = src[idx[j], :D] where idx[j] >= 0 (2-D row-pitched tensors)."""
    _lib.check(_lib.lib().b200q_ep_gather(src.data_ptr(), src.stride(0), idx.data_ptr(), idx.numel(), D,
                                          out.data_ptr(), out.stride(0), _stream_ptr(src.device)))
    return out


def pack_int4(codes: torch.Tensor, offset: int = 0) -> torch.Tensor:
    """4-bit codes [..., N] (int8 / uint8, one per byte) -> int32 [..., N/8]
    packed along N (nibble i of word j = column 8j + i).  offset 0: unsigned
    codes in [0, 15]; offset 8: signed int4 in [-8, 7] stored as q + 8 (use
    zero point 8).  Codes out of range set the device status bit."""
    if not codes.is_cuda:
        raise RuntimeError("b200q pack_int4 runs on CUDA tensors only")
    if codes.dtype not in (torch.int8, torch.uint8):
        raise TypeError("codes must be int8 or uint8")
    N = codes.shape[-1]
    c = _aligned(codes).reshape(-1, N)
    out = torch.empty(codes.shape[:-1] + (N // 8,), dtype=torch.int32, device=codes.device)
    ws = workspace(codes.device, 256)
    _lib.check(_lib.lib().b200q_pack_int4(c.data_ptr(), c.shape[0], N, offset, out.data_ptr(), ws.data_ptr(),
                                          _stream_ptr(codes.device)))
    return out


def silu_mul_fp8(y: torch.Tensor, codes: bool = False):
    """FUSED_SILU_REF: y [T, 2H] -> SiLU(gate) * up quantised per 128 columns
    to e4m3 and dequantised, fp32 [T, H].  With ``codes`` also returns the
    e4m3 codes (torch.float8_e4m3fn [T, H]) and scales (fp32 [T, H/128])."""
    if not y.is_cuda:
        raise RuntimeError("b200q silu_mul_fp8 runs on CUDA tensors only")
    T, H2 = y.shape
    H = H2 // 2
    y = _aligned(y)
    out = torch.empty((T, H), dtype=torch.float32, device=y.device)
    q = torch.empty((T, H), dtype=torch.uint8, device=y.device) if codes else None
    sc = torch.empty((T, H // 128), dtype=torch.float32, device=y.device) if codes else None
    _lib.check(_lib.lib().b200q_silu_mul_fp8(y.data_ptr(), T, H, _dtype_code(y.dtype), out.data_ptr(),
                                             q.data_ptr() if codes else None, sc.data_ptr() if codes else None,
                                             _stream_ptr(y.device)))
    if codes:
        return out, q.view(torch.float8_e4m3fn), sc
    return out


def lora_shrink(x: torch.Tensor, A: torch.Tensor, lora_ids: torch.Tensor) -> torch.Tensor:
    """lo [T, r] = x[t] . A[lora_ids[t]] per token (A [L, D, r]), x's dtype."""
    T, D = x.shape
    L, _, r = A.shape
    ids = lora_ids.to(torch.int64).contiguous()
    x, A = _aligned(x), _aligned(A.to(x.dtype))
    lo = torch.empty((T, r), dtype=x.dtype, device=x.device)
    ws = workspace(x.device, 256)
    _lib.check(_lib.lib().b200q_lora_shrink(x.data_ptr(), A.data_ptr(), ids.data_ptr(), T, D, r, L,
                                            _dtype_code(x.dtype), lo.data_ptr(), ws.data_ptr(),
                                            _stream_ptr(x.device)))
    return lo


def lora_expand_add(base: torch.Tensor, lo: torch.Tensor, B: torch.Tensor, lora_ids: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """y [T, N] = base + round(lo[t] . B[lora_ids[t]]) (B [L, r, N])."""
    T, N = base.shape
    L, r, _ = B.shape
    ids = lora_ids.to(torch.int64).contiguous()
    base, lo, B = _aligned(base), _aligned(lo), _aligned(B.to(base.dtype))
    y = out if out is not None else torch.empty_like(base)
    _lib.check(_lib.lib().b200q_lora_expand_add(base.data_ptr(), lo.data_ptr(), B.data_ptr(), ids.data_ptr(), T, r,
                                                N, L, _dtype_code(base.dtype), y.data_ptr(),
                                                _stream_ptr(base.device)))
    return y


def moe_gather(x: torch.Tensor, slot_token: torch.Tensor) -> torch.Tensor:
    x = _aligned(x)
    xg = torch.empty((slot_token.numel(), x.shape[1]), dtype=x.dtype, device=x.device)
    _lib.check(_lib.lib().b200q_moe_gather(x.data_ptr(), slot_token.data_ptr(), slot_token.numel(), x.shape[1],
                                           xg.data_ptr(), _stream_ptr(x.device)))
    return xg


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    gate, up = gate.contiguous(), up.contiguous()
    h = torch.empty_like(gate)
    _lib.check(_lib.lib().b200q_silu_mul(gate.data_ptr(), up.data_ptr(), h.data_ptr(), gate.numel(),
                                         _dtype_code(gate.dtype), _stream_ptr(gate.device)))
    return h


def moe_combine(ye: torch.Tensor, token_slot: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
    ye = ye.contiguous()
    T = token_slot.shape[0]
    y = torch.empty((T, ye.shape[1]), dtype=ye.dtype, device=ye.device)
    _lib.check(_lib.lib().b200q_moe_combine(ye.data_ptr(), token_slot.data_ptr(), gates.contiguous().data_ptr(),
                                            y.data_ptr(), T, ye.shape[1], _dtype_code(ye.dtype),
                                            _stream_ptr(ye.device)))
    return y


def set_weight_prefetch(enable: bool) -> bool:
    """Lets small-M W4A16 calls stream their weights while the previous kernel
    in the stream is still running (programmatic dependent launch).  Only valid
    when the kernel just before each call does not write that call's weights,
    scales or zeros.  Process-wide; returns the previous setting."""
    return bool(_lib.lib().b200q_set_weight_prefetch(1 if enable else 0))


def device_status(device: torch.device | None = None) -> int:
    """Reads and clears the device error word of this stream's workspace
    (synchronises the stream).  0 means no kernel reported an error."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = workspace(device, 4096)
    r = _lib.lib().b200q_workspace_status(ws.data_ptr(), _stream_ptr(device))
    if r < 0:
        _lib.check(r)
    if r > 0:
        ws.zero_()  # a kernel that gave up may have left split-K counters behind
    return r
