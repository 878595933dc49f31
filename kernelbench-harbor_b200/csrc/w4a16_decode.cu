// W4A16 group-quantised GEMM, small-M ("decode") path.
//
// y[M, N] = x[M, K] . W[K, N],  W[k, n] = (nib(k, n) - z[k/g, n]) * s[k/g, n]
// with the reference layout: qweight [K, N/8] int32 packed along N (nibble i
// of word [k, j] is column 8j+i), scales/zeros [K/g, N].  Same arithmetic as
// QUANT_REF.forward (generate_tasks.py:54-61): the dequantised weight is formed
// in the activation dtype exactly as the reference rounds it ((nib - z) exact,
// one rounding for * s), then multiplied with fp32 accumulation.
//
// Design (HBM-bound regime, M <= 32 per launch chunk; the library routes M >= 17 to the
// tcgen05 kernels, the allocation-free entry point uses it up to M = 32):
//  * The N axis is cut into 256-column strips (32 packed words = 128 B per K
//    row); the K axis of each strip into `splits` contiguous ranges so that
//    strips x splits ~= one CTA per SM (split-K).
//  * One producer warp streams 128-row stages with TMA (128B-swizzled) into a
//    6-deep shared-memory ring: the packed weight tile (16 KB), the x tile and
//    the scale/zero rows of the stage.  Eight consumer warps each take 128
//    columns x 32 rows of a stage.
//  * Consumers unpack nibbles with PRMT + LOP3 (magic-exponent int4 -> fp16),
//    subtract the zero point exactly, multiply by the scale, and feed
//    mma.sync m16n8k16 tiles with fp32 accumulators.  The tensor-core operand
//    map exploits that a GEMM may permute its reduction index: each thread
//    owns 4 consecutive K rows and two packed words, so one nibble position
//    of those words is exactly one B fragment -- no shuffles, no smem staging
//    of dequantised values.
//  * Split-K partials go to caller workspace slots; the last CTA of a strip
//    (atomic ticket, no spinning) sums the slots in a fixed order, writes y,
//    clears the slots and resets its ticket, so results are deterministic and
//    the workspace is left zeroed.
#include "common.cuh"

namespace b200q {
namespace decode {

constexpr int STRIP_WORDS = 32;
constexpr int STRIP_COLS = STRIP_WORDS * 8;  // 256
constexpr int KS = 128;                      // K rows per stage
constexpr int NCONS = 8;                     // consumer warps
constexpr int THREADS = (NCONS + 1) * 32;
constexpr int STAGES = 6;
constexpr int MAX_SPLITS = 16;  // split-K ranges per strip (bounded so the final sum stays in registers)
constexpr int HEADER_BYTES = 256;  // workspace: [status int | pad] then tickets then partials

template <int MT>
struct Layout {
  static constexpr int QW = KS * STRIP_WORDS * 4;  // 16 KB
  static constexpr int XBOX = 16 * 128;            // 16 rows x 64 k x 2 B
  static constexpr int X = MT * 2 * XBOX;
  static constexpr int SZ = 4 * STRIP_COLS * 2;  // up to 4 scale rows per stage (group 32)
  static constexpr int STAGE = QW + X + 2 * SZ;
  static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(STAGE % 1024 == 0, "stage must keep 1024-byte alignment for 128B swizzle");
  static_assert(NCONS * MT * 64 * 32 * 4 + 16 * MT * STRIP_COLS * 2 <= STAGES * STAGE,
                "reduction buffer and output tile must fit in the ring");
};

template <bool BF16>
struct DT;
template <>
struct DT<false> {
  using T = __half;
  using T2 = __half2;
};
template <>
struct DT<true> {
  using T = __nv_bfloat16;
  using T2 = __nv_bfloat162;
};

__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1, bool bf16) {
  if (!bf16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ uint32_t h2u(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
template <class T2>
__device__ __forceinline__ T2 u2h(uint32_t v) {
  return *reinterpret_cast<T2*>(&v);
}

// Dequantise the nibble pair at position t (0..7 of the word) held in the
// 16-bit halves of v (already PRMT-paired and shifted by 8 for t%4 >= 2).
// fp16: 0x6400|n is 1024+n; 0x6400|(n<<4) is 1024+16n, so the odd positions
// use an exact fma by 1/16.  Result is (n - z) * s with the reference's
// rounding (one rounding, in the multiply).
template <bool BF16>
__device__ __forceinline__ uint32_t dq(uint32_t v, int t, uint32_t zc, uint32_t s2);

template <>
__device__ __forceinline__ uint32_t dq<false>(uint32_t v, int t, uint32_t zc, uint32_t s2) {
  __half2 h;
  if ((t & 1) == 0) {
    h = __hsub2(u2h<__half2>(and_or(v, 0x000F000Fu, 0x64006400u)), u2h<__half2>(zc));
  } else {
    h = __hfma2(u2h<__half2>(and_or(v, 0x00F000F0u, 0x64006400u)), __half2half2(__float2half(0.0625f)),
                u2h<__half2>(zc));
  }
  return h2u(__hmul2_rn(h, u2h<__half2>(s2)));
}

// bf16: 0x4300|n is 128+n (ulp 1 in [128, 256)); no shifted form fits, so
// every position is brought down to bits 0..3 (callers pass v >> 4 for odd t).
template <>
__device__ __forceinline__ uint32_t dq<true>(uint32_t v, int t, uint32_t zc, uint32_t s2) {
  __nv_bfloat162 h = __hsub2(u2h<__nv_bfloat162>(and_or(v, 0x000F000Fu, 0x43004300u)), u2h<__nv_bfloat162>(zc));
  return h2u(__hmul2_rn(h, u2h<__nv_bfloat162>(s2)));
}

template <int MT, bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_decode_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                        const __grid_constant__ OutSet out, int M, int N, int K, int group, int strips, int splits,
                        int n_stages_total, uint8_t* __restrict__ ws) {
  using L = Layout<MT>;
  using T = typename DT<BF16>::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE);
  uint64_t* empty = full + STAGES;
  __shared__ int s_last;
  __shared__ int s_err;

  int* status = reinterpret_cast<int*>(ws);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = blockIdx.x / splits, split = blockIdx.x % splits;
  const int mchunk = blockIdx.y;
  const int st0 = (int)((long long)split * n_stages_total / splits);
  const int st1 = (int)((long long)(split + 1) * n_stages_total / splits);
  const int nst = st1 - st0;
  const int srows = group >= KS ? 1 : KS / group;
  const uint32_t stage_bytes = L::QW + L::X + 2u * srows * STRIP_COLS * 2u;
  int* tickets = reinterpret_cast<int*>(ws + HEADER_BYTES);
  float* partials = reinterpret_cast<float*>(ws + HEADER_BYTES + (((size_t)gridDim.y * strips * 4 + 255) & ~size_t(255)));

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCONS);
    }
    fence_barrier_init();
    s_err = 0;
    if (blockIdx.x == 0 && blockIdx.y == 0) peer_arrive(out);
  }
  if (warp == NCONS && lane == 0) {
    prefetch_tmap(&tm_qw);
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_s);
    prefetch_tmap(&tm_z);
  }
  __syncthreads();

  float acc[MT][16][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[mt][i][r] = 0.f;

  if (warp == NCONS) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      int it = 0;
      for (; it < nst; ++it) {
        const int s = it % STAGES;
        if (it >= STAGES) {
          if (!mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, status)) {
            atomicOr(&s_err, 1);
            break;
          }
        }
        uint8_t* st = smem + s * L::STAGE;
        const int k0 = (st0 + it) * KS;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        tma_load_2d_hint(st, &tm_qw, strip * STRIP_WORDS, k0, &full[s], pol_stream);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int row = mchunk * 16 * MT + mt * 16;
          tma_load_2d(st + L::QW + (mt * 2 + 0) * L::XBOX, &tm_x, k0, row, &full[s]);
          tma_load_2d(st + L::QW + (mt * 2 + 1) * L::XBOX, &tm_x, k0 + 64, row, &full[s]);
        }
        tma_load_2d(st + L::QW + L::X, &tm_s, strip * STRIP_COLS, k0 / group, &full[s]);
        tma_load_2d(st + L::QW + L::X + L::SZ, &tm_z, strip * STRIP_COLS, k0 / group, &full[s]);
      }
      // drain: never leave the CTA with bulk copies in flight
      const int issued = it;
      for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, status);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int g = lane >> 2, c = lane & 3;
    const int nh = warp & 1, kq = warp >> 1;
    for (int it = 0; it < nst; ++it) {
      const int s = it % STAGES;
      if (!mbar_wait(&full[s], (it / STAGES) & 1, status)) {
        atomicOr(&s_err, 1);
        break;
      }
      const uint8_t* st = smem + s * L::STAGE;
      // scale / zero of this warp's 32 rows (one group: group >= 32)
      const int srow = group >= KS ? 0 : (kq * 32) / group;
      const T* sp = reinterpret_cast<const T*>(st + L::QW + L::X) + srow * STRIP_COLS + nh * 128 + 16 * g;
      const T* zp = reinterpret_cast<const T*>(st + L::QW + L::X + L::SZ) + srow * STRIP_COLS + nh * 128 + 16 * g;
      uint32_t s2[16], zc[16];
      {
        const uint4 sv0 = reinterpret_cast<const uint4*>(sp)[0], sv1 = reinterpret_cast<const uint4*>(sp)[1];
        const uint4 zv0 = reinterpret_cast<const uint4*>(zp)[0], zv1 = reinterpret_cast<const uint4*>(zp)[1];
        const uint32_t sw[8] = {sv0.x, sv0.y, sv0.z, sv0.w, sv1.x, sv1.y, sv1.z, sv1.w};
        const uint32_t zw[8] = {zv0.x, zv0.y, zv0.z, zv0.w, zv1.x, zv1.y, zv1.z, zv1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          s2[2 * i] = prmt(sw[i], sw[i], 0x1010);
          s2[2 * i + 1] = prmt(sw[i], sw[i], 0x3232);
          if (!BF16) {
            // (z_even + 1024, -(z_odd + 64)) in one fma, then duplicate each half
            const __half2 zz = __hfma2(u2h<__half2>(zw[i]), __floats2half2_rn(1.f, -1.f),
                                       __floats2half2_rn(1024.f, -64.f));
            const uint32_t zu = h2u(zz);
            zc[2 * i] = prmt(zu, zu, 0x1010);
            zc[2 * i + 1] = prmt(zu, zu, 0x3232);
          } else {
            const __nv_bfloat162 zz = __hadd2(u2h<__nv_bfloat162>(zw[i]), __floats2bfloat162_rn(128.f, 128.f));
            const uint32_t zu = h2u(zz);
            zc[2 * i] = prmt(zu, zu, 0x1010);
            zc[2 * i + 1] = prmt(zu, zu, 0x3232);
          }
        }
      }
      const uint8_t* qw = st;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int r0 = kq * 32 + kk * 16 + 4 * c;
        uint2 wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = r0 + i;
          wv[i] = *reinterpret_cast<const uint2*>(qw + r * 128 + ((((nh * 4) + (g >> 1)) ^ (r & 7)) << 4) +
                                                  ((g & 1) << 3));
        }
        uint32_t a[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint8_t* xb = st + L::QW + (mt * 2 + (kq >> 1)) * L::XBOX;
          const int chunk = (kq & 1) * 4 + kk * 2 + (c >> 1);
          const uint2 lo = *reinterpret_cast<const uint2*>(xb + g * 128 + ((chunk ^ g) << 4) + ((c & 1) << 3));
          const uint2 hi =
              *reinterpret_cast<const uint2*>(xb + (g + 8) * 128 + ((chunk ^ g) << 4) + ((c & 1) << 3));
          a[mt][0] = lo.x;
          a[mt][1] = hi.x;
          a[mt][2] = lo.y;
          a[mt][3] = hi.y;
        }
#pragma unroll
        for (int om = 0; om < 2; ++om) {
          const uint32_t w0 = om ? wv[0].y : wv[0].x, w1 = om ? wv[1].y : wv[1].x;
          const uint32_t w2 = om ? wv[2].y : wv[2].x, w3 = om ? wv[3].y : wv[3].x;
          const uint32_t lo01 = prmt(w0, w1, 0x5410), hi01 = prmt(w0, w1, 0x7632);
          const uint32_t lo23 = prmt(w2, w3, 0x5410), hi23 = prmt(w2, w3, 0x7632);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            uint32_t v01 = t < 4 ? lo01 : hi01, v23 = t < 4 ? lo23 : hi23;
            if (!BF16) {
              if (t & 2) {
                v01 >>= 8;
                v23 >>= 8;
              }
            } else {
              const int sh = 4 * (t & 3);
              v01 >>= sh;
              v23 >>= sh;
            }
            const int ti = om * 8 + t;
            const uint32_t b0 = dq<BF16>(v01, t, zc[ti], s2[ti]);
            const uint32_t b1 = dq<BF16>(v23, t, zc[ti], s2[ti]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) mma_16816(acc[mt][ti], a[mt], b0, b1, BF16);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }

  __syncthreads();
  do {
    if (s_err) break;  // status word already records the timeout

    // ---------------------------------------------------------------- CTA reduction over the 4 K-quarters
    float* red = reinterpret_cast<float*>(smem);
    if (warp < NCONS) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int ti = 0; ti < 16; ++ti)
#pragma unroll
          for (int r = 0; r < 4; ++r) red[((warp * MT + mt) * 64 + ti * 4 + r) * 32 + lane] = acc[mt][ti][r];
    }
    __syncthreads();

    // The CTA's output block is walked in fragment order: internal index
    // i = ((nh * MT + mt) * 64 + e) * 32 + lane, e = tile * 4 + reg, which makes
    // the smem reads above lane-contiguous (conflict-free).  Workspace slots use
    // the same order; only the final store maps i to (row, column).
    const int rows_here = min(16 * MT, M - mchunk * 16 * MT);
    const int n_int = 2 * MT * 64 * 32;
    const size_t slot_elems = (size_t)n_int;
    const size_t strip_id = (size_t)mchunk * strips + strip;
    float* my_slot = partials + (strip_id * splits + split) * slot_elems;
    const int tid = threadIdx.x;
    auto row_of = [](int i) {  // row within the CTA block (0 .. 16*MT-1)
      const int ln = i & 31, e = (i >> 5) & 63;
      const int mt = (i >> 11) % MT;
      return mt * 16 + (ln >> 2) + ((e & 3) >> 1) * 8;
    };
    auto col_of = [](int i) {  // column within the 256-column strip
      const int ln = i & 31, e = (i >> 5) & 63, nh = (i >> 11) / MT;
      const int tile = e >> 2, r = e & 3, om = tile >> 3, t = tile & 7, c = ln & 3;
      return 8 * (nh * 16 + 2 * (2 * c + (r & 1)) + om) + t;
    };
    // the output block is assembled in shared memory (after the reduction
    // buffer) and leaves as whole rows of 16-byte chunks: coalesced in HBM and
    // few, large writes when the destinations are peers over NVLink
    T* tile = reinterpret_cast<T*>(smem + NCONS * MT * 64 * 32 * 4);
    auto write_rows = [&]() {
      for (int e = tid; e < rows_here * (STRIP_COLS / 8); e += THREADS) {
        const int row = e / (STRIP_COLS / 8), ch = e % (STRIP_COLS / 8);
        const int gcol = strip * STRIP_COLS + ch * 8;
        if (gcol >= N) continue;  // N % 32 == 0: a chunk is wholly inside or outside
        const uint4 v = *reinterpret_cast<const uint4*>(tile + row * STRIP_COLS + ch * 8);
        for (int o = 0; o < out.n; ++o)
          *reinterpret_cast<uint4*>(reinterpret_cast<T*>(out.y[o]) + (size_t)(mchunk * 16 * MT + row) * out.ldy +
                                    out.col0 + gcol) = v;
      }
    };
    if (splits == 1 && out.world > 1) {
      if (tid == 0 && !peer_wait_arrivals(out, status)) s_err = 1;
      __syncthreads();
      if (s_err) break;
    }
    for (int i = tid; i < n_int; i += THREADS) {
      const int row = row_of(i);
      if (row >= rows_here) continue;
      const int nh = (i >> 11) / MT, rest = i - nh * MT * 2048;
      float v = 0.f;
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) v += red[(kq * 2 + nh) * MT * 2048 + rest];
      if (splits == 1)
        tile[row * STRIP_COLS + col_of(i)] = (T)v;
      else
        my_slot[i] = v;
    }
    if (splits == 1) {
      __syncthreads();
      write_rows();
      break;
    }

    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&tickets[strip_id], 1) == splits - 1);
    __syncthreads();
    if (!s_last) break;
    __threadfence();
    if (out.world > 1) {
      if (tid == 0 && !peer_wait_arrivals(out, status)) s_err = 1;
      __syncthreads();
      if (s_err) break;
    }
    // all split slots of a float4 are loaded before any is summed (up to
    // MAX_SPLITS independent L2 reads in flight per thread), then added in slot
    // order, so the result does not depend on which CTA finished last.  The
    // slots are cleared after reading: every workspace byte this kernel wrote
    // goes back to zero (kernels sharing the workspace rely on zeroed memory).
    float4* slots = reinterpret_cast<float4*>(partials + strip_id * splits * slot_elems);
    const int slot4 = n_int / 4;
    for (int i4 = tid; i4 < slot4; i4 += THREADS) {
      const int i = i4 * 4;
      const int row = row_of(i);  // the 4 lanes of a float4 share a row
      if (row >= rows_here) continue;
      float4 part[MAX_SPLITS];
#pragma unroll
      for (int sp = 0; sp < MAX_SPLITS; ++sp)
        if (sp < splits) part[sp] = __ldcg(slots + sp * slot4 + i4);
#pragma unroll
      for (int sp = 0; sp < MAX_SPLITS; ++sp)
        if (sp < splits) __stcg(slots + sp * slot4 + i4, make_float4(0.f, 0.f, 0.f, 0.f));
      float4 v = part[0];
#pragma unroll
      for (int sp = 1; sp < MAX_SPLITS; ++sp)
        if (sp < splits) {
          v.x += part[sp].x;
          v.y += part[sp].y;
          v.z += part[sp].z;
          v.w += part[sp].w;
        }
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) tile[row * STRIP_COLS + col_of(i + q)] = (T)vv[q];
    }
    __syncthreads();
    write_rows();
    if (tid == 0) tickets[strip_id] = 0;  // leave the workspace zeroed for the next call
  } while (0);
  if (out.world > 1) {
    __syncthreads();
    if (threadIdx.x < 32) peer_finish(out, status);
  }
}

struct Plan {
  int mt, mchunks, strips, splits, n_stages;
  size_t ws_bytes;
};

Plan plan(int64_t M, int64_t N, int64_t K, int sms) {
  Plan p;
  p.mt = M <= 16 ? 1 : 2;
  p.mchunks = (int)((M + 16 * p.mt - 1) / (16 * p.mt));
  if (p.mchunks < 1) p.mchunks = 1;
  p.strips = (int)((N + STRIP_COLS - 1) / STRIP_COLS);
  p.n_stages = (int)((K + KS - 1) / KS);
  int sp = sms / (p.strips * p.mchunks);
  if (sp < 1) sp = 1;
  if (sp > p.n_stages) sp = p.n_stages;
  if (sp > MAX_SPLITS) sp = MAX_SPLITS;
  p.splits = sp;
  const size_t tickets = ((size_t)p.mchunks * p.strips * 4 + 255) & ~size_t(255);
  const size_t parts =
      p.splits > 1 ? (size_t)p.mchunks * p.strips * p.splits * (2 * p.mt * 64 * 32) * sizeof(float) : 0;
  p.ws_bytes = HEADER_BYTES + tickets + parts;
  return p;
}

template <int MT, bool BF16>
static int launch_t(const Plan& p, const CUtensorMap& qw, const CUtensorMap& x, const CUtensorMap& s,
                    const CUtensorMap& z, const OutSet& y, int M, int N, int K, int group, uint8_t* ws,
                    cudaStream_t stream) {
  auto kern = w4a16_decode_kernel<MT, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<MT>::SMEM);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(decode)");
  dim3 grid(p.strips * p.splits, p.mchunks);
  kern<<<grid, THREADS, Layout<MT>::SMEM, stream>>>(qw, x, s, z, y, M, N, K, group, p.strips, p.splits,
                                                     p.n_stages, ws);
  return check_cuda(cudaGetLastError(), "w4a16 decode launch");
}

}  // namespace decode

size_t w4a16_decode_ws_bytes(int64_t M, int64_t N, int64_t K, int device) {
  return decode::plan(M, N, K, num_sms(device)).ws_bytes;
}

int w4a16_decode(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& y,
                 int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream) {
  using namespace decode;
  const Plan p = plan(M, N, K, num_sms(-1));
  if (!workspace || workspace_bytes < p.ws_bytes)
    return fail(B200Q_ERR_WORKSPACE, "w4a16: workspace of " + std::to_string(p.ws_bytes) + " bytes required");
  const CUtensorMapDataType h16 = CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUtensorMap tqw, tx, ts, tz;
  const uint32_t srows = group >= KS ? 1 : (uint32_t)(KS / group);
  int rc;
  if ((rc = encode_2d(&tqw, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, N / 8, K, (uint64_t)N / 2, STRIP_WORDS, KS,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = encode_2d(&tx, h16, x, K, M, (uint64_t)K * 2, 64, 16, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = encode_2d(&ts, h16, scales, N, K / group, (uint64_t)N * 2, STRIP_COLS, srows,
                      CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = encode_2d(&tz, h16, zeros, N, K / group, (uint64_t)N * 2, STRIP_COLS, srows,
                      CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const bool bf = dtype == B200Q_DTYPE_BF16;
  if (p.mt == 1)
    return bf ? launch_t<1, true>(p, tqw, tx, ts, tz, y, (int)M, (int)N, (int)K, (int)group, ws, stream)
              : launch_t<1, false>(p, tqw, tx, ts, tz, y, (int)M, (int)N, (int)K, (int)group, ws, stream);
  return bf ? launch_t<2, true>(p, tqw, tx, ts, tz, y, (int)M, (int)N, (int)K, (int)group, ws, stream)
            : launch_t<2, false>(p, tqw, tx, ts, tz, y, (int)M, (int)N, (int)K, (int)group, ws, stream);
}

}  // namespace b200q
