// W4A16 group-quantised GEMM on tcgen05 as a persistent kernel with a hybrid
// data-parallel / stream-K schedule: the compute-bound ("prefill", M >= 17)
// path of the plain GEMM.
//
// Same arithmetic, tile and warp roles as the per-tile kernel (w4a16_tc.cu):
// y[M, N] = x[M, K] . W[K, N] with W[k, n] = (nib(k, n) - z[k/g, n]) * s[k/g, n]
// dequantised on the fly into the MN-major B operand, fp32 accumulation in
// TMEM.  What differs is the work distribution.  One CTA runs per SM (G of
// them).  Tiles are 128 or 256 rows (MB = 1 or 2 row blocks sharing each
// dequantised weight tile; 256 from M = 129 on: half the dequantisation per
// FLOP) by 256 columns, numbered with the column tile fastest.  Whole waves of
// tiles are data-parallel: CTA c takes tiles c, c + G, ... from k = 0, so the
// CTAs of a wave stream the same rows of x at the same time and share them in
// L2.  The remaining tiles' 64-deep K stages form one linear space of units
// that the CTAs split evenly (stream-K), so every SM ends at about the same
// time whatever the tile count.
//
// A CTA walks its work as segments (tile, K range).  A segment covering the
// whole K range stores its tile directly.  A split tile has one owner, the
// CTA whose range holds its k = 0 stage (for which the tile is the last
// segment of its range), and contributors, the following CTAs (for each of
// which it is the first segment).  A contributor writes its fp32 partial tile
// to its slot in the workspace and publishes it (a counter per tile).  The
// owner, after its own part, waits for its contributors, pulls each partial
// into shared memory (free by then: its last stages are consumed) with one
// bulk copy per pass and adds it into its TMEM accumulator, in ascending CTA
// order (ascending K, so the result does not depend on timing), zeroing the
// slot behind it, then stores the tile.  Contributors publish before they
// wait on anything and all G <= #SMs CTAs are resident, so the owners' waits
// always end; they are bounded anyway.  Owners reset their tiles' counters:
// the workspace is left zeroed.
//
// TMEM holds one accumulator set (MB x 256 columns); the MMA of the next
// segment waits until the epilogue warps have read the previous one out.
#include "w4a16_dq.cuh"

namespace b200q {
namespace sk {

using namespace tc;

constexpr int MIN_UNITS = 8;  // K stages per CTA at least (tiny problems use fewer CTAs)
constexpr int MAX_SPLIT = 8;  // CTAs sharing one tile, on average at most (the owner adds the others serially)

constexpr int MAX_SEGS = 64;  // segments of one CTA (data-parallel rounds + stream-K pieces)

// Work partition.  Tiles [0, dp_rounds * G) are data-parallel: CTA c takes
// tiles c, c + G, ... whole.  The remaining tiles' K stages form a linear
// unit space of U units that the first Gs CTAs split evenly (stream-K).
struct Part {
  long long U;  // stream-K units = (tiles - dp_rounds * G) * nk
  int tiles_m, tiles_n, nk, G, Gs, dp_rounds;
};

__device__ __forceinline__ long long ubeg(const Part& p, int c) {
  return c >= p.Gs ? p.U : (long long)c * p.U / p.Gs;
}

// CTA whose stream-K range holds unit u (0 <= u < U)
__device__ __forceinline__ int cta_of(const Part& p, long long u) {
  int c = (int)(u * p.Gs / p.U);
  while (c + 1 < p.Gs && ubeg(p, c + 1) <= u) ++c;
  while (c > 0 && ubeg(p, c) > u) --c;
  return c;
}

struct Seg {
  int t, kb, ke;
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

__host__ __device__ constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

template <bool BF16, int MB>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_sk_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wq,
                    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                    const __grid_constant__ OutSet out, int M, int N, int K, int group, const Part p,
                    uint8_t* __restrict__ ws) {
  using T = typename DT<BF16>::T;
  using C = Cfg<MB>;
  constexpr int R = MB * BM;  // rows per tile
  constexpr size_t SLOT_FLOATS = (size_t)R * BN;
  constexpr int SX = C::SX, SW = C::SW, S2 = C::S2;
  constexpr uint32_t X_BYTES = C::X_BYTES, OFF_X = C::OFF_X, OFF_B = C::OFF_B, OFF_WQ = C::OFF_WQ,
                     OFF_S = C::OFF_S, OFF_Z = C::OFF_Z, OFF_BAR = C::OFF_BAR;
  static_assert((2 * SX + 2 * SW + 2 * S2 + 2) * 8 + 4 <= 256, "barrier area");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* x_full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* x_empty = x_full + SX;
  uint64_t* w_full = x_empty + SX;
  uint64_t* w_empty = w_full + SW;
  uint64_t* b_full = w_empty + SW;
  uint64_t* b_empty = b_full + S2;
  uint64_t* acc_full = b_empty + S2;
  uint64_t* tmem_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 1);
  __shared__ int s_err;
  __shared__ int s_nseg;
  __shared__ Seg s_seg[MAX_SEGS];

  int* status = reinterpret_cast<int*>(ws);
  const int tiles = p.tiles_m * p.tiles_n;
  uint32_t* tilec = reinterpret_cast<uint32_t*>(ws + HEADER_BYTES);  // [tiles]: partials published
  float* slots = reinterpret_cast<float*>(ws + HEADER_BYTES + align256((size_t)tiles * 4));  // [G][R x BN]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int dp_tiles = p.dp_rounds * p.G;
  const int srows = group >= BK ? 1 : BK / group;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SX; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], NDQ);
    }
    for (int j = 0; j < S2; ++j) {
      mbar_init(&b_full[j], NDQ);
      mbar_init(&b_empty[j], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(tmem_empty, NDQ);
    fence_barrier_init();
    s_err = 0;
    if (c == 0) peer_arrive(out);
    // this CTA's segments: its data-parallel tiles, then its stream-K range
    int n = 0;
    for (int r = 0; r < p.dp_rounds; ++r) s_seg[n++] = Seg{c + r * p.G, 0, p.nk};
    const long long u0 = ubeg(p, c), u1 = ubeg(p, c + 1);
    for (long long u = u0; u < u1 && n < MAX_SEGS;) {
      const int tr = (int)(u / p.nk), kb = (int)(u - (long long)tr * p.nk);
      const int ke = (int)min((long long)p.nk, kb + (u1 - u));
      s_seg[n++] = Seg{dp_tiles + tr, kb, ke};
      u += ke - kb;
    }
    s_nseg = n;
  }
  if (warp == W_PROD && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_wq);
    prefetch_tmap(&tm_s);
    prefetch_tmap(&tm_z);
  }
  __syncwarp();
  if (warp == W_MMA) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == W_PROD) {
    // ---------------------------------------------------------------- weight producer
    if (lane == 0) {
      const uint32_t stage_tx = WQ_BYTES + 2u * srows * BN * 2u;
      int s = 0, n = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int i = 0; ok && i < s_nseg; ++i) {
        const Seg g = s_seg[i];
        const int n0 = (g.t % p.tiles_n) * BN;
        for (int k = g.kb; k < g.ke; ++k, ++n) {
          if (n >= SW && !mbar_wait(&w_empty[s], ph ^ 1, status)) {
            s_err = 1;
            ok = false;
            break;
          }
          const int kb = k * BK;
          mbar_arrive_expect_tx(&w_full[s], stage_tx);
          tma_load_2d(smem + OFF_WQ + s * WQ_BYTES, &tm_wq, n0 / 8, kb, &w_full[s]);
          tma_load_2d(smem + OFF_S + s * SZ_BYTES, &tm_s, n0, kb / group, &w_full[s]);
          tma_load_2d(smem + OFF_Z + s * SZ_BYTES, &tm_z, n0, kb / group, &w_full[s]);
          if (++s == SW) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == W_XPROD) {
    // ---------------------------------------------------------------- activation producer
    if (lane == 0) {
      int s = 0, n = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int i = 0; ok && i < s_nseg; ++i) {
        const Seg g = s_seg[i];
        const int m0 = (g.t / p.tiles_n) * R;
        for (int k = g.kb; k < g.ke; ++k, ++n) {
          if (n >= SX && !mbar_wait(&x_empty[s], ph ^ 1, status)) {
            s_err = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[s], X_BYTES);
#pragma unroll
          for (int mb = 0; mb < MB; ++mb)
            tma_load_2d(smem + OFF_X + s * X_BYTES + mb * XB_BYTES, &tm_x, k * BK, m0 + mb * BM, &x_full[s]);
          if (++s == SX) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == W_MMA) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BM, BN, BF16 ? 1 : 0, /*a_mn=*/0, /*b_mn=*/1);
      int sx = 0, sb = 0, sg = 0;
      uint32_t phx = 0, phb = 0;
      bool ok = true;
      for (; ok && sg < s_nseg; ++sg) {
        const Seg g = s_seg[sg];
        if (sg > 0 && !mbar_wait(tmem_empty, (sg - 1) & 1, status)) {
          s_err = 1;
          break;
        }
        tc_fence_after();
        for (int k = g.kb; k < g.ke; ++k) {
          if (!mbar_wait(&x_full[sx], phx, status) || !mbar_wait(&b_full[sb], phb, status)) {
            s_err = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xa = smem_u32(smem + OFF_X + sx * X_BYTES);
          const uint32_t bb = smem_u32(smem + OFF_B + sb * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // A: K-major, 8-row groups 1024 B apart; B: MN-major, 64-column
            // atoms 1024 B apart, 8-row K groups 4096 B apart
            const uint64_t bd = smem_desc(bb + kk * 8192, 1024, 4096, 2);
#pragma unroll
            for (int mb = 0; mb < MB; ++mb) {
              const uint64_t ad = smem_desc(xa + mb * XB_BYTES + kk * 32, 16, 1024, 2);
              tc_mma_f16_ss(tmem + mb * BN, ad, bd, idesc, (k != g.kb) || (kk != 0));
            }
          }
          tc_commit(&x_empty[sx]);
          tc_commit(&b_empty[sb]);
          if (++sx == SX) {
            sx = 0;
            phx ^= 1;
          }
          if (++sb == S2) {
            sb = 0;
            phb ^= 1;
          }
        }
        if (ok) tc_commit(acc_full);
      }
    }
  } else {
    // ---------------------------------------------------------------- dequantise + epilogue
    const int dw = warp - W_DQ0;
    const int dq_tid = threadIdx.x - W_DQ0 * 32;
    const int nb = lane >> 3, ch = lane & 7;
    const int rr = dw & 7;  // row within each 8-row group
    static_assert(WPR == 2, "a thread's words i < WORDS/2 lie in K rows 0..31 of the stage, the rest in 32..63");
    const uint32_t* wq_t = reinterpret_cast<const uint32_t*>(smem + OFF_WQ) + (rr + 8 * (dw >> 3)) * 32 + lane;
    constexpr int WQ_ROW_STEP = 8 * WPR * 32;
    uint8_t* b_t = smem + OFF_B + ((dw >> 3) * 4 + nb) * 1024 + rr * 128 + ((ch ^ rr) << 4);
    const int qd = warp & 3;   // TMEM lane quadrant this warp may access
    const int part = dw >> 2;  // which of the NDQ/4 column ranges of this quadrant
    constexpr int COLS = MB * BN / (NDQ / 4);
    const int acc = (part * COLS) / BN;
    const int trow = acc * BM + qd * 32 + lane;  // row within the tile
    const uint32_t tl = tmem + ((uint32_t)(qd * 32) << 16);
    // Every epilogue warp runs the same sequence of named barriers whatever
    // happens: after an error (a timed-out wait, recorded in s_err) the loops
    // keep their shape and skip the work.
    volatile int* err = &s_err;
    bool peers_ready = out.world <= 1;
    auto wait_peers = [&]() {  // before the first store into a (peer) output
      if (peers_ready) return;
      if (dq_tid == 0 && !*err && !peer_wait_arrivals(out, status)) *err = 1;
      named_barrier_sync(1, NDQ * 32);
      peers_ready = true;
    };

    int s = 0, j = 0, n = 0, sg = 0;
    uint32_t ph_w = 0, ph_b = 0;
    for (; sg < s_nseg; ++sg) {
      const Seg g = s_seg[sg];
      for (int k = g.kb; k < g.ke; ++k, ++n) {
        const bool good = !*err && mbar_wait(&w_full[s], ph_w, status) &&
                          (n < S2 || mbar_wait(&b_empty[j], ph_b ^ 1, status));
        if (good) {
        const uint8_t* srow0 = smem + OFF_S + s * SZ_BYTES;
        const uint8_t* zrow0 = smem + OFF_Z + s * SZ_BYTES;
        const ColQ q0 = load_colq<BF16>(srow0, zrow0, lane);
        const ColQ q1 = srows > 1 ? load_colq<BF16>(srow0 + BN * 2, zrow0 + BN * 2, lane) : q0;
        const uint32_t* wq = wq_t + s * (WQ_BYTES / 4);
        uint32_t wv[WORDS];
#pragma unroll
        for (int i = 0; i < WORDS; ++i) wv[i] = wq[i * WQ_ROW_STEP];
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_empty[s]);
        uint8_t* bt = b_t + j * B_BYTES;
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
          const uint4 v = dequant_word<BF16>(wv[i], i >= WORDS / 2 ? q1 : q0);
          *reinterpret_cast<uint4*>(bt + i * (WPR * 4 * 1024)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b_full[j]);
        } else {
          *err = 1;
        }
        if (++s == SW) {
          s = 0;
          ph_w ^= 1;
        }
        if (++j == S2) {
          j = 0;
          ph_b ^= 1;
        }
      }

      // ---- epilogue of the segment.  A whole-K segment stores its tile.  A
      // segment that starts past k = 0 (the first of this CTA's range) is a
      // contributor: it writes its fp32 partial to this CTA's slot and
      // publishes it.  A segment from k = 0 that stops short (the last of the
      // range) is the tile's owner: it waits for its contributors (the next
      // CTAs, for which the tile was the first segment), adds their partials
      // into its TMEM accumulator one after another in ascending CTA order
      // (ascending K), zeroes the slots it consumed and stores the tile.
      const bool contrib = g.kb != 0;
      const bool owner = g.kb == 0 && g.ke < p.nk;
      const int c_hi = owner ? cta_of(p, (long long)(g.t - dp_tiles) * p.nk + p.nk - 1) : c;
      if (!contrib) wait_peers();
      if (owner) {
        if (dq_tid == 0 && !*err) {
          const uint64_t t0 = globaltimer();
          for (uint32_t it = 0; ld_acquire_gpu(tilec + g.t) < (uint32_t)(c_hi - c); ++it) {
            if ((it & 63) == 63 && globaltimer() - t0 > B200Q_WAIT_NS) {
              atomicOr(status, B200Q_DEV_ERR_TIMEOUT);
              *err = 1;
              break;
            }
            __nanosleep(64);
          }
          tilec[g.t] = 0;  // every contributor has published: the counter is free for the next call
        }
        named_barrier_sync(1, NDQ * 32);
      }
      const bool acc_ok = !*err && mbar_wait(acc_full, sg & 1, status);
      if (!acc_ok) *err = 1;
      if (acc_ok) tc_fence_after();
      if (acc_ok && !*err) {
        const int m0 = (g.t / p.tiles_n) * R, n0 = (g.t % p.tiles_n) * BN;
#pragma unroll 1
        for (int c0 = 0; c0 < COLS; c0 += 32) {
          const int ocol = (part * COLS + c0) % BN;
          uint32_t r[32];
          tmem_ld32(tl + acc * BN + ocol, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) v[(q & ~7) | slot_col(q & 7)] = __uint_as_float(r[q]);
          // slot layout: element (row, col) at ((col / 4) * R + row) * 4 + col % 4:
          // a warp's 32 rows of one 4-column group are 512 contiguous bytes
          const size_t so = (size_t)(ocol >> 2) * R + trow;
          if (contrib) {
            float4* slot = reinterpret_cast<float4*>(slots + (size_t)c * SLOT_FLOATS) + so;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              __stcg(slot + (size_t)q * R, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
            continue;
          }
          for (int cq = c + 1; cq <= c_hi; ++cq) {  // owner: contributors in ascending K order
            float4* slot = reinterpret_cast<float4*>(slots + (size_t)cq * SLOT_FLOATS) + so;
            float4 a4[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) a4[q] = __ldcg(slot + (size_t)q * R);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              v[4 * q] += a4[q].x;
              v[4 * q + 1] += a4[q].y;
              v[4 * q + 2] += a4[q].z;
              v[4 * q + 3] += a4[q].w;
              __stcg(slot + (size_t)q * R, make_float4(0.f, 0.f, 0.f, 0.f));  // leave the slot zeroed
            }
          }
          const int row = m0 + trow, col = n0 + ocol;
          if (row < M && col < N) {
            uint32_t pk[16];
#pragma unroll
            for (int q = 0; q < 16; ++q)
              pk[q] = BF16 ? as_u32(__floats2bfloat162_rn(v[2 * q], v[2 * q + 1]))
                           : as_u32(__floats2half2_rn(v[2 * q], v[2 * q + 1]));
            for (int o = 0; o < out.n; ++o) {
              uint4* dst =
                  reinterpret_cast<uint4*>(reinterpret_cast<T*>(out.y[o]) + (size_t)row * out.ldy + out.col0 + col);
#pragma unroll
              for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_empty);
      if (contrib) {
        named_barrier_sync(1, NDQ * 32);  // every partial store of the CTA issued
        if (dq_tid == 0 && !*err) {
          __threadfence();
          atomicAdd(tilec + g.t, 1u);
        }
      }
    }
  }

  // every role above diverged within its warp (one elected lane): reconverge
  // before the CTA-wide barrier, which counts whole warps
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (out.world > 1) {
    __syncthreads();
    if (threadIdx.x < 32) peer_finish(out, status);
  }
}

struct Plan {
  int mb, segs;
  Part part;
  size_t ws_bytes;
};

Plan plan(int64_t M, int64_t N, int64_t K, int sms) {
  Plan pl;
  pl.mb = M > BM ? 2 : 1;
  Part& p = pl.part;
  p.tiles_m = (int)((M + BM * pl.mb - 1) / (BM * pl.mb));
  p.tiles_n = (int)((N + BN - 1) / BN);
  p.nk = (int)((K + BK - 1) / BK);
  const long long tiles = (long long)p.tiles_m * p.tiles_n;
  if (tiles >= sms) {
    // whole waves data-parallel (concurrent CTAs start every tile at k = 0,
    // sharing x in L2); the remainder stream-K over all SMs, or folded into
    // the last wave's stream-K when it is a small fraction of a wave
    p.G = sms;
    p.dp_rounds = (int)(tiles / sms);
    const long long rem = tiles - (long long)p.dp_rounds * sms;
    if (rem > 0 && rem * 4 < sms) --p.dp_rounds;
  } else {
    long long g = tiles * p.nk / MIN_UNITS;
    if (g > tiles * MAX_SPLIT) g = tiles * MAX_SPLIT;
    if (g < 1) g = 1;
    if (g > sms) g = sms;
    p.G = (int)g;
    p.dp_rounds = 0;
  }
  const long long sk_tiles = tiles - (long long)p.dp_rounds * p.G;
  p.U = sk_tiles * p.nk;
  long long gs = p.U / MIN_UNITS;
  if (gs > sk_tiles * MAX_SPLIT) gs = sk_tiles * MAX_SPLIT;
  if (gs > p.G) gs = p.G;
  if (gs < 1) gs = 1;
  p.Gs = (int)gs;
  pl.segs = p.dp_rounds + (p.U > 0 ? (int)((p.U / p.Gs + p.nk - 1) / p.nk) + 2 : 0);
  const size_t slot = (size_t)pl.mb * BM * BN * 4;
  pl.ws_bytes = HEADER_BYTES + align256((size_t)tiles * 4) + (size_t)p.Gs * slot;
  return pl;
}

}  // namespace sk

size_t w4a16_sk_ws_bytes(int64_t M, int64_t N, int64_t K, int device) {
  return sk::plan(M, N, K, num_sms(device)).ws_bytes;
}

int w4a16_sk(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& out,
             int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace, size_t workspace_bytes,
             cudaStream_t stream) {
  using namespace sk;
  const Plan pl = plan(M, N, K, num_sms(-1));
  if (pl.segs > MAX_SEGS) return fail(B200Q_ERR_SHAPE, "w4a16: M x N too large for the tile schedule");
  if (!workspace || workspace_bytes < pl.ws_bytes)
    return fail(B200Q_ERR_WORKSPACE, "w4a16: workspace of " + std::to_string(pl.ws_bytes) + " bytes required");
  const CUtensorMapDataType h16 = CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const uint32_t srows = group >= BK ? 1 : (uint32_t)(BK / group);
  CUtensorMap tx, twq, ts, tz;
  int rc;
  if ((rc = encode_2d(&tx, h16, x, K, M, (uint64_t)K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = encode_2d(&twq, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, N / 8, K, (uint64_t)N / 2, BN / 8, BK,
                      CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = encode_2d(&ts, h16, scales, N, K / group, (uint64_t)N * 2, BN, srows, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = encode_2d(&tz, h16, zeros, N, K / group, (uint64_t)N * 2, BN, srows, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  const bool bf = dtype == B200Q_DTYPE_BF16;
  auto kern = pl.mb == 2 ? (bf ? w4a16_sk_kernel<true, 2> : w4a16_sk_kernel<false, 2>)
                         : (bf ? w4a16_sk_kernel<true, 1> : w4a16_sk_kernel<false, 1>);
  const uint32_t smem = pl.mb == 2 ? Cfg<2>::SMEM : Cfg<1>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(w4a16 stream-K)");
  kern<<<pl.part.G, THREADS, smem, stream>>>(tx, twq, ts, tz, out, (int)M, (int)N, (int)K, (int)group, pl.part,
                                              reinterpret_cast<uint8_t*>(workspace));
  return check_cuda(cudaGetLastError(), "w4a16 stream-K launch");
}

}  // namespace b200q
