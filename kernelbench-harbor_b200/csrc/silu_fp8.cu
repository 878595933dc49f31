// Fused SiLU * mul + per-group dynamic fp8 (e4m3) quantisation: the
// FUSED_SILU_REF module (generate_tasks.py:321-348), the activation step
// between a MoE's gate/up and down projections when the down projection runs
// in fp8.
//
// y [T, 2H] = concat(gate, up) in fp16/bf16.  act = SiLU(gate) * up in fp32
// (SiLU(g) = g / (1 + exp(-g))); per group of 128 consecutive columns of a
// row: scale = max(amax(|act|) / 448, 1e-12), q = e4m3(clamp(act / scale,
// -448, 448)) rounded to nearest even; outputs: the dequantised q * scale in
// fp32 (what the reference module returns), and / or the e4m3 codes and the
// fp32 scales [T, H/128] for an fp8 consumer.  One warp per group, 4
// columns per lane, the amax a warp-shuffle reduction: one pass over y.
#include <cuda_fp8.h>

#include "common.cuh"

namespace b200q {
namespace {

constexpr int GROUP = 128;
constexpr float FP8_MAX = 448.f;

template <class T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <class T>
__global__ void silu_mul_fp8_kernel(const T* __restrict__ y, int T_, int H, float* __restrict__ out,
                                    uint8_t* __restrict__ q_out, float* __restrict__ s_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = H / GROUP;
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + warp;  // (row, group)
  if (gid >= (long long)T_ * G) return;
  const int t = (int)(gid / G), g = (int)(gid % G);
  const T* gate = y + (size_t)t * 2 * H + g * GROUP + lane * 4;
  const T* up = gate + H;
  float a[4], amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float gv = to_f<T>(gate[i]);
    a[i] = gv / (1.f + expf(-gv)) * to_f<T>(up[i]);
    amax = fmaxf(amax, fabsf(a[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(amax / FP8_MAX, 1e-12f);
  uint32_t codes = 0;
  float d[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float v = fminf(fmaxf(a[i] / scale, -FP8_MAX), FP8_MAX);
    const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
    codes |= (uint32_t)c << (8 * i);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(c, __NV_E4M3);
    d[i] = __half2float(__half(hr)) * scale;
  }
  const size_t o = (size_t)t * H + g * GROUP + lane * 4;
  if (out) *reinterpret_cast<float4*>(out + o) = make_float4(d[0], d[1], d[2], d[3]);
  if (q_out) *reinterpret_cast<uint32_t*>(q_out + o) = codes;
  if (s_out && lane == 0) s_out[(size_t)t * G + g] = scale;
}

}  // namespace
}  // namespace b200q

extern "C" int b200q_silu_mul_fp8(const void* y, int64_t T, int64_t H, int dtype, float* out_dequant,
                                  uint8_t* q_out, float* scales_out, void* stream) {
  using namespace b200q;
  if (T < 0 || H <= 0 || H % GROUP) return fail(B200Q_ERR_SHAPE, "silu_mul_fp8: H must be a positive multiple of 128");
  if (T > (1ll << 30) || H > (1ll << 28)) return fail(B200Q_ERR_SHAPE, "silu_mul_fp8: size too large");
  if (T == 0) return B200Q_OK;
  if (!y || (!out_dequant && !q_out && !scales_out)) return fail(B200Q_ERR_SHAPE, "silu_mul_fp8: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(y) & 7) || (reinterpret_cast<uintptr_t>(out_dequant) & 15) ||
      (reinterpret_cast<uintptr_t>(q_out) & 3))
    return fail(B200Q_ERR_ALIGN, "silu_mul_fp8: y 8-byte, out 16-byte, q 4-byte aligned");
  const long long groups = T * (H / GROUP);
  const int warps = 8;
  const unsigned blocks = (unsigned)((groups + warps - 1) / warps);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == B200Q_DTYPE_FP16)
    silu_mul_fp8_kernel<__half><<<blocks, warps * 32, 0, st>>>(reinterpret_cast<const __half*>(y), (int)T, (int)H,
                                                               out_dequant, q_out, scales_out);
  else if (dtype == B200Q_DTYPE_BF16)
    silu_mul_fp8_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(y), (int)T, (int)H, out_dequant, q_out, scales_out);
  else
    return fail(B200Q_ERR_UNSUPPORTED, "silu_mul_fp8: dtype must be fp16 or bf16");
  return check_cuda(cudaGetLastError(), "silu_mul_fp8 launch");
}
