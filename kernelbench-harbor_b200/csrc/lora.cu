// Per-token gathered LoRA of the multi-LoRA quantised linear (LORA_REF,
// generate_tasks.py:397-424): y[t] = base[t] + (x[t] . A[id_t]) . B[id_t],
// with base = x . dequant(W) from the W4A16 kernels.  Shapes x [T, D],
// A [L, D, r], B [L, r, N], ids [T] (int64, the reference's lora_ids), r <= 64.
// Rounding as the reference module: lo = x . A rounded to the activation type
// (fp32 accumulation), lo . B rounded, then base + that rounded once.
//
// shrink: one CTA per token; warp w sums a slice of D, lane l columns l and
// l + 32 of r (A rows are r contiguous values), a shared-memory sum over the
// warps in fixed order.  expand: one thread per output column, the token's r
// values of lo in shared memory, B rows read coalesced along N.  An adapter
// id outside [0, L) sets B200Q_DEV_ERR_BOUNDS and leaves that token's row of
// lo zero / y equal to base.
#include "common.cuh"

namespace b200q {
namespace {

constexpr int MAX_R = 64;
constexpr int SHRINK_WARPS = 8;

template <class T>
__device__ __forceinline__ float tf(T v);
template <>
__device__ __forceinline__ float tf<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float tf<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <class T>
__device__ __forceinline__ T ft(float v);
template <>
__device__ __forceinline__ __half ft<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 ft<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <class T>
__global__ void lora_shrink_kernel(const T* __restrict__ x, const T* __restrict__ A, const int64_t* __restrict__ ids,
                                   int D, int r, int L, T* __restrict__ lo, int* status) {
  __shared__ float part[SHRINK_WARPS][MAX_R];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < L;
  if (!ok && threadIdx.x == 0 && status) atomicOr(status, B200Q_DEV_ERR_BOUNDS);
  float a0 = 0.f, a1 = 0.f;
  if (ok) {
    const T* xr = x + (size_t)t * D;
    const T* Ar = A + (size_t)id * D * r;
    const int d0 = warp * D / SHRINK_WARPS, d1 = (warp + 1) * D / SHRINK_WARPS;
    for (int d = d0; d < d1; ++d) {
      const float xv = tf<T>(xr[d]);
      if (lane < r) a0 = fmaf(xv, tf<T>(Ar[(size_t)d * r + lane]), a0);
      if (lane + 32 < r) a1 = fmaf(xv, tf<T>(Ar[(size_t)d * r + lane + 32]), a1);
    }
  }
  part[warp][lane] = a0;
  part[warp][lane + 32] = a1;
  __syncthreads();
  for (int c = threadIdx.x; c < r; c += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < SHRINK_WARPS; ++w) s += part[w][c];
    lo[(size_t)t * r + c] = ft<T>(ok ? s : 0.f);
  }
}

template <class T>
__global__ void lora_expand_add_kernel(const T* __restrict__ base, const T* __restrict__ lo,
                                       const T* __restrict__ B, const int64_t* __restrict__ ids, int r, int N, int L,
                                       T* __restrict__ y) {
  __shared__ float l_s[MAX_R];
  const int t = blockIdx.y;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < L;
  for (int c = threadIdx.x; c < r; c += blockDim.x) l_s[c] = tf<T>(lo[(size_t)t * r + c]);
  __syncthreads();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float acc = 0.f;
  if (ok) {
    const T* Bc = B + (size_t)id * r * N + n;
    for (int c = 0; c < r; ++c) acc = fmaf(l_s[c], tf<T>(Bc[(size_t)c * N]), acc);
  }
  const float b = tf<T>(base[(size_t)t * N + n]);
  y[(size_t)t * N + n] = ft<T>(b + tf<T>(ft<T>(acc)));
}

}  // namespace
}  // namespace b200q

extern "C" {

int b200q_lora_shrink(const void* x, const void* A, const int64_t* lora_ids, int64_t T, int64_t D, int64_t r,
                      int64_t L, int dtype, void* lo, void* workspace, void* stream) {
  using namespace b200q;
  if (T < 0 || D <= 0 || r <= 0 || r > MAX_R || L <= 0)
    return fail(B200Q_ERR_SHAPE, "lora_shrink: need T >= 0, D > 0, 0 < r <= 64, L > 0");
  if (T > (1ll << 30) || D * r * L > (1ll << 40)) return fail(B200Q_ERR_SHAPE, "lora_shrink: size too large");
  if (T == 0) return B200Q_OK;
  if (!x || !A || !lora_ids || !lo) return fail(B200Q_ERR_SHAPE, "lora_shrink: null pointer argument");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int* status = reinterpret_cast<int*>(workspace);
  if (dtype == B200Q_DTYPE_FP16)
    lora_shrink_kernel<__half><<<(unsigned)T, SHRINK_WARPS * 32, 0, st>>>(
        reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(A), lora_ids, (int)D, (int)r, (int)L,
        reinterpret_cast<__half*>(lo), status);
  else if (dtype == B200Q_DTYPE_BF16)
    lora_shrink_kernel<__nv_bfloat16><<<(unsigned)T, SHRINK_WARPS * 32, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(A), lora_ids, (int)D,
        (int)r, (int)L, reinterpret_cast<__nv_bfloat16*>(lo), status);
  else
    return fail(B200Q_ERR_UNSUPPORTED, "lora_shrink: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "lora_shrink launch");
}

int b200q_lora_expand_add(const void* base, const void* lo, const void* B, const int64_t* lora_ids, int64_t T,
                          int64_t r, int64_t N, int64_t L, int dtype, void* y, void* stream) {
  using namespace b200q;
  if (T < 0 || N <= 0 || r <= 0 || r > MAX_R || L <= 0)
    return fail(B200Q_ERR_SHAPE, "lora_expand_add: need T >= 0, N > 0, 0 < r <= 64, L > 0");
  if (T > 65535 || N > (1ll << 30)) return fail(B200Q_ERR_SHAPE, "lora_expand_add: size too large");
  if (T == 0) return B200Q_OK;
  if (!base || !lo || !B || !lora_ids || !y) return fail(B200Q_ERR_SHAPE, "lora_expand_add: null pointer argument");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((N + 255) / 256), (unsigned)T);
  if (dtype == B200Q_DTYPE_FP16)
    lora_expand_add_kernel<__half><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __half*>(base), reinterpret_cast<const __half*>(lo), reinterpret_cast<const __half*>(B),
        lora_ids, (int)r, (int)N, (int)L, reinterpret_cast<__half*>(y));
  else if (dtype == B200Q_DTYPE_BF16)
    lora_expand_add_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(base), reinterpret_cast<const __nv_bfloat16*>(lo),
        reinterpret_cast<const __nv_bfloat16*>(B), lora_ids, (int)r, (int)N, (int)L,
        reinterpret_cast<__nv_bfloat16*>(y));
  else
    return fail(B200Q_ERR_UNSUPPORTED, "lora_expand_add: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "lora_expand_add launch");
}

}  // extern "C"
