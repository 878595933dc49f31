// Quantised top-2 mixture-of-experts: routing, token permutation, SiLU.mul and
// the gated combine.  The expert GEMMs are the W4A16 kernels of this library.
//
// Reference semantics (FUSED_QMOE_REF / MOE_REF, generate_tasks.py:171-178,
// 368-378, SiLU.mul of FUSED_SILU_REF :336-337):
//   probs = softmax(logits.float());  topv, topi = probs.topk(2)
//   gates = (topv / topv.sum()).to(x.dtype)
//   h_e   = (silu(gate_e.float()) * up_e.float()).to(x.dtype)
//   y[t]  = sum_k  out_{topi[t,k]}[t] * gates[t,k]      (x.dtype products, one sum)
// Selection compares the logits (softmax is monotonic; distinct fp16 logits give
// distinct fp32 probabilities); equal logits: the lower expert index wins.
//
// Permutation: the routing kernel (one CTA, deterministic) writes, per expert e,
// the tokens routed to it in ascending token order into slots
// [offsets[e], offsets[e+1]), plus each token's two slot numbers.  Experts then
// run on contiguous row blocks, and the combine reads each token's two rows.
#include <algorithm>

#include "common.cuh"

namespace b200q {
namespace moe {

constexpr int ROUTE_THREADS = 1024;
constexpr int MAX_EXPERTS = 256;

template <class T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <class T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <class T>
__global__ void __launch_bounds__(ROUTE_THREADS, 1)
    route_kernel(const T* __restrict__ logits, int T_, int E, int32_t* __restrict__ topi, T* __restrict__ gates,
                 int32_t* __restrict__ offsets, int32_t* __restrict__ slot_token, int32_t* __restrict__ token_slot) {
  __shared__ int s_count[MAX_EXPERTS];
  __shared__ int s_base[MAX_EXPERTS];
  __shared__ int s_warp[ROUTE_THREADS / 32];
  __shared__ int s_total;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  for (int e = tid; e < E; e += ROUTE_THREADS) s_count[e] = 0;
  __syncthreads();
  // pass 1: top-2 per token, gates, expert counts
  for (int t = tid; t < T_; t += ROUTE_THREADS) {
    const T* l = logits + (size_t)t * E;
    float v0 = -INFINITY, v1 = -INFINITY;
    int i0 = 0, i1 = 1;
    for (int e = 0; e < E; ++e) {
      const float v = to_f<T>(l[e]);
      if (v > v0) {
        v1 = v0;
        i1 = i0;
        v0 = v;
        i0 = e;
      } else if (v > v1) {
        v1 = v;
        i1 = e;
      }
    }
    if (i1 == i0) i1 = i0 == 0 ? 1 : 0;  // E >= 2 guaranteed by the caller; all -inf rows
    // softmax of the two selected entries over all E (max is v0)
    float sum = 0.f;
    for (int e = 0; e < E; ++e) sum += expf(to_f<T>(l[e]) - v0);
    const float p0 = 1.f / sum, p1 = expf(v1 - v0) / sum;
    const float tot = p0 + p1;
    topi[2 * t] = i0;
    topi[2 * t + 1] = i1;
    gates[2 * t] = from_f<T>(p0 / tot);
    gates[2 * t + 1] = from_f<T>(p1 / tot);
    atomicAdd(&s_count[i0], 1);
    atomicAdd(&s_count[i1], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      s_base[e] = acc;
      acc += s_count[e];
    }
    offsets[E] = acc;
  }
  __syncthreads();
  // pass 2: stable slots (ascending token order within each expert): for each
  // expert, a block-wide exclusive scan of "token t is routed to e" per chunk
  for (int t0 = 0; t0 < T_; t0 += ROUTE_THREADS) {
    const int t = t0 + tid;
    const bool valid = t < T_;
    const int a = valid ? topi[2 * t] : -1, b = valid ? topi[2 * t + 1] : -1;
    for (int e = 0; e < E; ++e) {
      const bool f = (a == e) || (b == e);
      const unsigned m = __ballot_sync(0xffffffffu, f);
      if (lane == 0) s_warp[wid] = __popc(m);
      __syncthreads();
      if (tid == 0) {
        int acc = 0;
        for (int w = 0; w < ROUTE_THREADS / 32; ++w) {
          const int c = s_warp[w];
          s_warp[w] = acc;
          acc += c;
        }
        s_total = acc;
      }
      __syncthreads();
      if (f) {
        const int slot = s_base[e] + s_warp[wid] + __popc(m & ((1u << lane) - 1u));
        slot_token[slot] = t;
        token_slot[2 * t + (a == e ? 0 : 1)] = slot;
      }
      __syncthreads();
      if (tid == 0) s_base[e] += s_total;
      __syncthreads();
    }
  }
}

__global__ void gather_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ slot_token, int nslots,
                              int row16, uint4* __restrict__ xg) {
  const int slot = blockIdx.x;
  if (slot >= nslots) return;
  const uint4* src = x + (size_t)slot_token[slot] * row16;
  uint4* dst = xg + (size_t)slot * row16;
  for (int i = threadIdx.x; i < row16; i += blockDim.x) dst[i] = src[i];
}

template <class T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ h, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float a = to_f<T>(g[i]);
    h[i] = from_f<T>(a / (1.f + expf(-a)) * to_f<T>(u[i]));
  }
}

template <class T>
__global__ void combine_kernel(const T* __restrict__ ye, const int32_t* __restrict__ token_slot,
                               const T* __restrict__ gates, T* __restrict__ y, int D) {
  const int t = blockIdx.x;
  const int s0 = token_slot[2 * t], s1 = token_slot[2 * t + 1];
  const float g0 = to_f<T>(gates[2 * t]), g1 = to_f<T>(gates[2 * t + 1]);
  // 8 values (16 bytes) per thread and step; D % 8 == 0
  const uint4* a = reinterpret_cast<const uint4*>(ye + (size_t)s0 * D);
  const uint4* b = reinterpret_cast<const uint4*>(ye + (size_t)s1 * D);
  uint4* o = reinterpret_cast<uint4*>(y + (size_t)t * D);
  for (int q = threadIdx.x; q < D / 8; q += blockDim.x) {
    const uint4 va = a[q], vb = b[q];
    const T* pa = reinterpret_cast<const T*>(&va);
    const T* pb = reinterpret_cast<const T*>(&vb);
    uint4 vo;
    T* po = reinterpret_cast<T*>(&vo);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // x.dtype products (one rounding each), then their sum rounded once
      const float p0 = to_f<T>(from_f<T>(to_f<T>(pa[i]) * g0));
      const float p1 = to_f<T>(from_f<T>(to_f<T>(pb[i]) * g1));
      po[i] = from_f<T>(p0 + p1);
    }
    o[q] = vo;
  }
}

}  // namespace moe
}  // namespace b200q

extern "C" {

int b200q_moe_route(const void* logits, int64_t T, int64_t E, int dtype, int32_t* topi, void* gates,
                    int32_t* offsets, int32_t* slot_token, int32_t* token_slot, void* stream) {
  using namespace b200q;
  if (T < 0 || E < 2 || E > moe::MAX_EXPERTS)
    return fail(B200Q_ERR_SHAPE, "moe_route: need T >= 0 and 2 <= E <= 256");
  if (dtype != B200Q_DTYPE_FP16 && dtype != B200Q_DTYPE_BF16)
    return fail(B200Q_ERR_UNSUPPORTED, "moe_route: dtype must be fp16 or bf16");
  if (T > (1ll << 30)) return fail(B200Q_ERR_SHAPE, "moe_route: too many tokens");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == B200Q_DTYPE_FP16)
    moe::route_kernel<__half><<<1, moe::ROUTE_THREADS, 0, st>>>(
        reinterpret_cast<const __half*>(logits), (int)T, (int)E, topi, reinterpret_cast<__half*>(gates), offsets,
        slot_token, token_slot);
  else
    moe::route_kernel<__nv_bfloat16><<<1, moe::ROUTE_THREADS, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits), (int)T, (int)E, topi,
        reinterpret_cast<__nv_bfloat16*>(gates), offsets, slot_token, token_slot);
  return check_cuda(cudaGetLastError(), "moe_route launch");
}

int b200q_moe_gather(const void* x, const int32_t* slot_token, int64_t nslots, int64_t D, void* xg, void* stream) {
  using namespace b200q;
  if (nslots < 0 || D <= 0 || D % 8) return fail(B200Q_ERR_SHAPE, "moe_gather: D must be a positive multiple of 8");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(xg)) & 15)
    return fail(B200Q_ERR_ALIGN, "moe_gather: pointers must be 16-byte aligned");
  if (nslots == 0) return B200Q_OK;
  moe::gather_kernel<<<(unsigned)nslots, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(x), slot_token, (int)nslots, (int)(D / 8), reinterpret_cast<uint4*>(xg));
  return check_cuda(cudaGetLastError(), "moe_gather launch");
}

int b200q_silu_mul(const void* gate, const void* up, void* h, int64_t n, int dtype, void* stream) {
  using namespace b200q;
  if (n < 0) return fail(B200Q_ERR_SHAPE, "silu_mul: n must be >= 0");
  if (n == 0) return B200Q_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
  if (dtype == B200Q_DTYPE_FP16)
    moe::silu_mul_kernel<__half><<<blocks, 256, 0, st>>>(reinterpret_cast<const __half*>(gate),
                                                          reinterpret_cast<const __half*>(up),
                                                          reinterpret_cast<__half*>(h), (size_t)n);
  else if (dtype == B200Q_DTYPE_BF16)
    moe::silu_mul_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(gate),
                                                                 reinterpret_cast<const __nv_bfloat16*>(up),
                                                                 reinterpret_cast<__nv_bfloat16*>(h), (size_t)n);
  else
    return fail(B200Q_ERR_UNSUPPORTED, "silu_mul: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "silu_mul launch");
}

int b200q_moe_combine(const void* ye, const int32_t* token_slot, const void* gates, void* y, int64_t T, int64_t D,
                      int dtype, void* stream) {
  using namespace b200q;
  if (T < 0 || D <= 0 || D % 8) return fail(B200Q_ERR_SHAPE, "moe_combine: T >= 0, D a positive multiple of 8");
  if ((reinterpret_cast<uintptr_t>(ye) | reinterpret_cast<uintptr_t>(y)) & 15)
    return fail(B200Q_ERR_ALIGN, "moe_combine: ye and y must be 16-byte aligned");
  if (T == 0) return B200Q_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == B200Q_DTYPE_FP16)
    moe::combine_kernel<__half><<<(unsigned)T, 128, 0, st>>>(reinterpret_cast<const __half*>(ye), token_slot,
                                                              reinterpret_cast<const __half*>(gates),
                                                              reinterpret_cast<__half*>(y), (int)D);
  else if (dtype == B200Q_DTYPE_BF16)
    moe::combine_kernel<__nv_bfloat16><<<(unsigned)T, 128, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(ye), token_slot, reinterpret_cast<const __nv_bfloat16*>(gates),
        reinterpret_cast<__nv_bfloat16*>(y), (int)D);
  else
    return fail(B200Q_ERR_UNSUPPORTED, "moe_combine: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "moe_combine launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Expert-parallel exchange helpers (the benchmark's expert-parallel MoE; the
// reference MoE is single-GPU, generate_tasks.py:368-378).  With P ranks,
// E / P experts per rank and C row slots per (source, destination) pair:
//   ep_pack     fills this rank's send buffer [P * C, D + 8] from its routed
//               tokens: slot d * C + j holds the j-th row routed to rank d
//               (expert-grouped order of moe_route), column D the destination
//               expert's local index as a small integer in the activation type
//               (-1: empty slot); pair_slot[t, k] = the slot of token t's k-th row;
//   ep_regroup  (one CTA) orders the received rows [P * C, D + 8] stably by
//               local expert: loc_offsets [E/P + 1], src[j] = received row at
//               grouped position j (-1 past the last), row_pos[r] = grouped
//               position of received row r (-1: empty slot);
//   ep_gather   dst[j, :D] = src[idx[j], :D] for idx[j] >= 0, any row pitches.
namespace b200q {
namespace moe {

template <class T>
__global__ void ep_pack_kernel(const uint4* __restrict__ x, int row16, const int32_t* __restrict__ offsets,
                               const int32_t* __restrict__ slot_token, const int32_t* __restrict__ token_slot, int P,
                               int C, int epr, T* __restrict__ send, int send_pitch, int32_t* __restrict__ pair_slot) {
  const int r = blockIdx.x;
  const int d = r / C, li = r % C;
  const int base = offsets[d * epr], cnt = offsets[(d + 1) * epr] - base;
  T* row = send + (size_t)r * send_pitch;
  const int D = row16 * 8;
  if (li >= cnt) {
    if (threadIdx.x < 8) row[D + threadIdx.x] = from_f<T>(threadIdx.x == 0 ? -1.f : 0.f);
    return;
  }
  const int i = base + li;
  const int t = slot_token[i];
  int e = d * epr;
  while (e + 1 < (d + 1) * epr && offsets[e + 1] <= i) ++e;
  const uint4* src = x + (size_t)t * row16;
  uint4* dst = reinterpret_cast<uint4*>(row);
  for (int q = threadIdx.x; q < row16; q += blockDim.x) dst[q] = src[q];
  if (threadIdx.x < 8) row[D + threadIdx.x] = from_f<T>(threadIdx.x == 0 ? (float)(e - d * epr) : 0.f);
  if (threadIdx.x == 0) pair_slot[2 * t + (token_slot[2 * t] == i ? 0 : 1)] = r;
}

template <class T>
__global__ void __launch_bounds__(1024, 1)
    ep_regroup_kernel(const T* __restrict__ recv, int pitch, int D, int R, int epr, int32_t* __restrict__ loc_offsets,
                      int32_t* __restrict__ src, int32_t* __restrict__ row_pos) {
  __shared__ int s_cnt[MAX_EXPERTS], s_base[MAX_EXPERTS], s_warp[32][65];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < epr; e += blockDim.x) s_cnt[e] = 0;
  for (int j = tid; j < R; j += blockDim.x) src[j] = -1;
  __syncthreads();
  auto eid_of = [&](int r) { return (int)rintf(to_f<T>(recv[(size_t)r * pitch + D])); };
  for (int r = tid; r < R; r += blockDim.x) {
    const int e = eid_of(r);
    if (e >= 0 && e < epr) atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < epr; ++e) {
      s_base[e] = acc;
      loc_offsets[e] = acc;
      acc += s_cnt[e];
    }
    loc_offsets[epr] = acc;
  }
  __syncthreads();
  // stable positions, 1024 rows at a time, experts in blocks of 64
  for (int r0 = 0; r0 < R; r0 += blockDim.x) {
    const int r = r0 + tid;
    const int e = r < R ? eid_of(r) : -1;
    int pos = -1;
    for (int e0 = 0; e0 < epr; e0 += 64) {
      const int ne = min(64, epr - e0);
      for (int k = 0; k < ne; ++k) {
        const unsigned m = __ballot_sync(0xffffffffu, e == e0 + k);
        if (lane == 0) s_warp[warp][k] = __popc(m);
        if (e == e0 + k) pos = __popc(m & ((1u << lane) - 1u));  // rank within the warp
      }
      __syncthreads();
      if (tid < ne) {  // exclusive prefix over the warps, per expert
        int acc = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
          const int v = s_warp[w][tid];
          s_warp[w][tid] = acc;
          acc += v;
        }
        s_cnt[e0 + tid] = acc;  // rows of this chunk for the expert
      }
      __syncthreads();
      if (e >= e0 && e < e0 + ne) pos += s_base[e] + s_warp[warp][e - e0];
      __syncthreads();
      if (tid < ne) s_base[e0 + tid] += s_cnt[e0 + tid];
      __syncthreads();
    }
    if (r < R) {
      row_pos[r] = (e >= 0 && e < epr) ? pos : -1;
      if (e >= 0 && e < epr) src[pos] = r;
    }
  }
}

__global__ void ep_gather_kernel(const uint4* __restrict__ src, int src_pitch16, const int32_t* __restrict__ idx,
                                 int row16, uint4* __restrict__ dst, int dst_pitch16) {
  const int j = blockIdx.x;
  const int s = idx[j];
  if (s < 0) return;
  const uint4* a = src + (size_t)s * src_pitch16;
  uint4* b = dst + (size_t)j * dst_pitch16;
  for (int q = threadIdx.x; q < row16; q += blockDim.x) b[q] = a[q];
}

}  // namespace moe
}  // namespace b200q

extern "C" {

int b200q_ep_pack(const void* x, int64_t T, int64_t D, int dtype, const int32_t* offsets, const int32_t* slot_token,
                  const int32_t* token_slot, int64_t E, int64_t P, int64_t C, void* send, int32_t* pair_slot,
                  void* stream) {
  using namespace b200q;
  if (T < 0 || D <= 0 || D % 8 || P < 1 || E % P || E > moe::MAX_EXPERTS || C < 0 || P * C > (1ll << 30))
    return fail(B200Q_ERR_SHAPE, "ep_pack: need D % 8 == 0, E % P == 0, E <= 256");
  if (C < 2 * T) return fail(B200Q_ERR_SHAPE, "ep_pack: need C >= 2 T (every pair may go to one rank)");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send)) & 15)
    return fail(B200Q_ERR_ALIGN, "ep_pack: x and send must be 16-byte aligned");
  if (P * C == 0) return B200Q_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int epr = (int)(E / P), pitch = (int)D + 8;
  if (dtype == B200Q_DTYPE_FP16)
    moe::ep_pack_kernel<__half><<<(unsigned)(P * C), 128, 0, st>>>(
        reinterpret_cast<const uint4*>(x), (int)(D / 8), offsets, slot_token, token_slot, (int)P, (int)C, epr,
        reinterpret_cast<__half*>(send), pitch, pair_slot);
  else if (dtype == B200Q_DTYPE_BF16)
    moe::ep_pack_kernel<__nv_bfloat16><<<(unsigned)(P * C), 128, 0, st>>>(
        reinterpret_cast<const uint4*>(x), (int)(D / 8), offsets, slot_token, token_slot, (int)P, (int)C, epr,
        reinterpret_cast<__nv_bfloat16*>(send), pitch, pair_slot);
  else
    return fail(B200Q_ERR_UNSUPPORTED, "ep_pack: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "ep_pack launch");
}

int b200q_ep_regroup(const void* recv, int64_t R, int64_t D, int dtype, int64_t n_local, int32_t* loc_offsets,
                     int32_t* src, int32_t* row_pos, void* stream) {
  using namespace b200q;
  if (R < 0 || D <= 0 || D % 8 || n_local < 1 || n_local > moe::MAX_EXPERTS || R > (1ll << 30))
    return fail(B200Q_ERR_SHAPE, "ep_regroup: need D % 8 == 0 and 1 <= n_local <= 256");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == B200Q_DTYPE_FP16)
    moe::ep_regroup_kernel<__half><<<1, 1024, 0, st>>>(reinterpret_cast<const __half*>(recv), (int)D + 8, (int)D,
                                                       (int)R, (int)n_local, loc_offsets, src, row_pos);
  else if (dtype == B200Q_DTYPE_BF16)
    moe::ep_regroup_kernel<__nv_bfloat16><<<1, 1024, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(recv),
                                                              (int)D + 8, (int)D, (int)R, (int)n_local, loc_offsets,
                                                              src, row_pos);
  else
    return fail(B200Q_ERR_UNSUPPORTED, "ep_regroup: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "ep_regroup launch");
}

int b200q_ep_gather(const void* src, int64_t src_pitch, const int32_t* idx, int64_t n, int64_t D, void* dst,
                    int64_t dst_pitch, void* stream) {
  using namespace b200q;
  if (n < 0 || D <= 0 || D % 8 || src_pitch % 8 || dst_pitch % 8 || src_pitch < D || dst_pitch < D)
    return fail(B200Q_ERR_SHAPE, "ep_gather: D and pitches must be multiples of 8 elements, pitches >= D");
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15)
    return fail(B200Q_ERR_ALIGN, "ep_gather: pointers must be 16-byte aligned");
  if (n == 0) return B200Q_OK;
  moe::ep_gather_kernel<<<(unsigned)n, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), (int)(src_pitch / 8), idx, (int)(D / 8), reinterpret_cast<uint4*>(dst),
      (int)(dst_pitch / 8));
  return check_cuda(cudaGetLastError(), "ep_gather launch");
}

}  // extern "C"
