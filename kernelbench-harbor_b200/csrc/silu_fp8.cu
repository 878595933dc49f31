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
// fp32 scales [T, H/128] for an fp8 consumer.  One half-warp per group, 8
// columns per lane (16-byte loads), two groups in flight per half-warp, the
// amax a shuffle reduction over the half-warp: one pass over y.
#include <cuda_fp8.h>

#include <type_traits>

#include "common.cuh"

namespace b200q {
namespace {

constexpr int GROUP = 128;
constexpr float FP8_MAX = 448.f;

template <class T>
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (std::is_same<T, __half>::value) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    } else {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
}

// One half-warp per (row, 128-column group), 8 columns per lane (16-byte
// loads); each half-warp handles GPT groups with all loads issued first.
constexpr int GPT = 2;

template <class T>
__global__ void __launch_bounds__(256) silu_mul_fp8_kernel(const T* __restrict__ y, int T_, int H,
                                                           float* __restrict__ out, uint8_t* __restrict__ q_out,
                                                           float* __restrict__ s_out) {
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int G = H / GROUP;
  const long long total = (long long)T_ * G;
  const long long g0 = ((long long)blockIdx.x * (blockDim.x >> 4) + hw) * GPT;  // first (row, group)
  uint4 gv[GPT], uv[GPT];
#pragma unroll
  for (int k = 0; k < GPT; ++k) {
    const long long gid = g0 + k;
    if (gid < total) {
      const int t = (int)(gid / G), g = (int)(gid % G);
      const T* gate = y + (size_t)t * 2 * H + g * GROUP + l * 8;
      gv[k] = __ldg(reinterpret_cast<const uint4*>(gate));
      uv[k] = __ldg(reinterpret_cast<const uint4*>(gate + H));
    }
  }
#pragma unroll
  for (int k = 0; k < GPT; ++k) {
    const long long gid = g0 + k;
    const bool live = gid < total;  // the whole half-warp agrees
    float gf[8], uf[8], a[8], amax = 0.f;
    if (live) {
      unpack8<T>(gv[k], gf);
      unpack8<T>(uv[k], uf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] = gf[i] / (1.f + expf(-gf[i])) * uf[i];
        amax = fmaxf(amax, fabsf(a[i]));
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (!live) continue;
    const int t = (int)(gid / G), g = (int)(gid % G);
    const float scale = fmaxf(amax / FP8_MAX, 1e-12f);
    uint32_t codes[2] = {0u, 0u};
    float d[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = fminf(fmaxf(a[i] / scale, -FP8_MAX), FP8_MAX);
      const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
      codes[i >> 2] |= (uint32_t)c << (8 * (i & 3));
      const __half_raw hr = __nv_cvt_fp8_to_halfraw(c, __NV_E4M3);
      d[i] = __half2float(__half(hr)) * scale;
    }
    const size_t o = (size_t)t * H + g * GROUP + l * 8;
    if (out) {
      reinterpret_cast<float4*>(out + o)[0] = make_float4(d[0], d[1], d[2], d[3]);
      reinterpret_cast<float4*>(out + o)[1] = make_float4(d[4], d[5], d[6], d[7]);
    }
    if (q_out) *reinterpret_cast<uint2*>(q_out + o) = make_uint2(codes[0], codes[1]);
    if (s_out && l == 0) s_out[(size_t)t * G + g] = scale;
  }
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
  if ((reinterpret_cast<uintptr_t>(y) & 15) || (reinterpret_cast<uintptr_t>(out_dequant) & 15) ||
      (reinterpret_cast<uintptr_t>(q_out) & 7))
    return fail(B200Q_ERR_ALIGN, "silu_mul_fp8: y and out 16-byte, q 8-byte aligned");
  const long long groups = T * (H / GROUP);
  const int warps = 8;  // 16 half-warps of GPT groups each per block
  const long long per_block = 2ll * warps * GPT;
  const unsigned blocks = (unsigned)((groups + per_block - 1) / per_block);
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
