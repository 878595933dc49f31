// Shared pieces of the tcgen05 W4A16 kernel (w4a16_tc.cu): tile and ring
// geometry, the per-column scale / zero constants and the LOP3
// magic-exponent dequantisation of one packed word.
#pragma once
#include "common.cuh"

namespace b200q {
namespace tc {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int NDQ = 16;         // dequantising (and epilogue) warps
constexpr int WPR = NDQ / 8;    // warps per row-in-group position
constexpr int WORDS = 8 / WPR;  // packed words per thread per stage
constexpr int W_PROD = 0, W_MMA = 1, W_XPROD = 2, W_DQ0 = 3;  // warp roles
constexpr int THREADS = (W_DQ0 + NDQ) * 32;
constexpr uint32_t XB_BYTES = BM * BK * 2;         // one 128-row x box: 16 KB
constexpr uint32_t WQ_BYTES = BK * (BN / 8) * 4;   // 8 KB
constexpr uint32_t SZ_BYTES = 2 * BN * 2;          // up to 2 scale rows per stage (group 32)
constexpr uint32_t B_BYTES = BK * BN * 2;          // 32 KB
constexpr int HEADER_BYTES = 256;
constexpr int MAX_SPLITS = 8;  // portable cluster size

#ifndef B200Q_TC1_SX
#define B200Q_TC1_SX 4
#endif
#ifndef B200Q_TC1_SW
#define B200Q_TC1_SW 6
#endif
#ifndef B200Q_TC1_S2
#define B200Q_TC1_S2 3
#endif

// MB = number of 128-row blocks of x per CTA sharing each dequantised B tile
// (1: 128 x 256 tile, 256 TMEM columns; 2: 256 x 256 tile, all 512 columns).
template <int MB>
struct Cfg {
  static constexpr int SX = MB == 1 ? B200Q_TC1_SX : 3;  // x ring (held until the MMAs of the stage complete)
  static constexpr int SW = MB == 1 ? B200Q_TC1_SW : 4;  // packed-weight + scale/zero ring (held until dequantised)
  static constexpr int S2 = MB == 1 ? B200Q_TC1_S2 : 2;  // dequantised-B ring
  static constexpr uint32_t X_BYTES = MB * XB_BYTES;
  static constexpr uint32_t OFF_X = 0;
  static constexpr uint32_t OFF_B = OFF_X + SX * X_BYTES;
  static constexpr uint32_t OFF_WQ = OFF_B + S2 * B_BYTES;
  static constexpr uint32_t OFF_S = OFF_WQ + SW * WQ_BYTES;
  static constexpr uint32_t OFF_Z = OFF_S + SW * SZ_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_Z + SW * SZ_BYTES;
  static constexpr uint32_t SMEM = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TMEM_COLS = MB * BN;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert((2 * SX + 2 * SW + 2 * S2 + 1) * 8 + 4 <= 256, "barrier area");
};

template <bool BF16>
struct DT;
template <>
struct DT<false> {
  using T = __half;
};
template <>
struct DT<true> {
  using T = __nv_bfloat16;
};

__device__ __forceinline__ uint32_t as_u32(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
__device__ __forceinline__ __nv_bfloat162 as_b2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// Per-thread constants for the 8 columns of one packed word in one group:
// scale pairs and zero-point terms in the (0,4)(1,5)(2,6)(3,7) pair order.
struct ColQ {
  uint32_t s[4], z[4];
};

template <bool BF16>
__device__ __forceinline__ ColQ load_colq(const uint8_t* s_row, const uint8_t* z_row, int lane) {
  const uint4 sv = *reinterpret_cast<const uint4*>(s_row + lane * 16);
  const uint4 zv = *reinterpret_cast<const uint4*>(z_row + lane * 16);
  ColQ q;
  q.s[0] = prmt(sv.x, sv.z, 0x5410);
  q.s[1] = prmt(sv.x, sv.z, 0x7632);
  q.s[2] = prmt(sv.y, sv.w, 0x5410);
  q.s[3] = prmt(sv.y, sv.w, 0x7632);
  const uint32_t z04 = prmt(zv.x, zv.z, 0x5410), z15 = prmt(zv.x, zv.z, 0x7632);
  const uint32_t z26 = prmt(zv.y, zv.w, 0x5410), z37 = prmt(zv.y, zv.w, 0x7632);
  if (!BF16) {
    const __half2 k1024 = __float2half2_rn(1024.f);
    const __half2 m1 = __float2half2_rn(-1.f), m64 = __float2half2_rn(-64.f);
    q.z[0] = as_u32(__hadd2(as_h2(z04), k1024));   // 1024 + z
    q.z[1] = as_u32(__hfma2(as_h2(z15), m1, m64));  // -(64 + z)
    q.z[2] = as_u32(__hadd2(as_h2(z26), k1024));
    q.z[3] = as_u32(__hfma2(as_h2(z37), m1, m64));
  } else {
    const __nv_bfloat162 k128 = __float2bfloat162_rn(128.f);
    q.z[0] = as_u32(__hadd2(as_b2(z04), k128));
    q.z[1] = as_u32(__hadd2(as_b2(z15), k128));
    q.z[2] = as_u32(__hadd2(as_b2(z26), k128));
    q.z[3] = as_u32(__hadd2(as_b2(z37), k128));
  }
  return q;
}

// Packed f16x2 / bf16x2 arithmetic on 32-bit registers (no conversions
// between the vector types and integer registers).
__device__ __forceinline__ uint32_t sub_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t fma_f16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t mul_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One packed word -> 8 dequantised values in pair order (n0,n4)(n1,n5)(n2,n6)(n3,n7).
// fp16: 0x6400|n is 1024+n and 0x6400|(n<<4) is 1024+16n, so the odd positions
// use an exact fma by 1/16; (n - z) is exact and the multiply by s is the one
// rounding, as in the reference.  bf16: 0x4300|n is 128+n.
template <bool BF16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, const ColQ& q) {
  uint4 o;
  if (!BF16) {
    const uint32_t r16 = 0x2C002C00u;  // (1/16, 1/16) in f16
    const uint32_t w8 = w >> 8;
    o.x = mul_f16x2(sub_f16x2(and_or(w, 0x000F000Fu, 0x64006400u), q.z[0]), q.s[0]);
    o.y = mul_f16x2(fma_f16x2(and_or(w, 0x00F000F0u, 0x64006400u), r16, q.z[1]), q.s[1]);
    o.z = mul_f16x2(sub_f16x2(and_or(w8, 0x000F000Fu, 0x64006400u), q.z[2]), q.s[2]);
    o.w = mul_f16x2(fma_f16x2(and_or(w8, 0x00F000F0u, 0x64006400u), r16, q.z[3]), q.s[3]);
  } else {
    o.x = mul_bf16x2(sub_bf16x2(and_or(w, 0x000F000Fu, 0x43004300u), q.z[0]), q.s[0]);
    o.y = mul_bf16x2(sub_bf16x2(and_or(w >> 4, 0x000F000Fu, 0x43004300u), q.z[1]), q.s[1]);
    o.z = mul_bf16x2(sub_bf16x2(and_or(w >> 8, 0x000F000Fu, 0x43004300u), q.z[2]), q.s[2]);
    o.w = mul_bf16x2(sub_bf16x2(and_or(w >> 12, 0x000F000Fu, 0x43004300u), q.z[3]), q.s[3]);
  }
  return o;
}

// B-operand slot -> actual column within each group of 8
__device__ __forceinline__ int slot_col(int p) { return ((p & 1) << 2) | (p >> 1); }

}  // namespace tc
}  // namespace b200q
