// W4A16 group-quantised GEMM on the 5th-generation tensor cores (tcgen05):
// the compute-bound ("prefill", M >= 17) path.
//
// y[M, N] = x[M, K] . W[K, N],  W[k, n] = (nib(k, n) - z[k/g, n]) * s[k/g, n],
// reference layout (QUANT_REF, generate_tasks.py:45-61): qweight [K, N/8]
// int32 packed along N, scales / zeros [K/g, N].  The dequantised weight is
// formed exactly as the reference rounds it ((nib - z) exact, one rounding in
// the multiply by s, in the activation dtype) and the product accumulates in
// fp32 in tensor memory.
//
// One CTA computes a 128 x 256 or 256 x 256 output tile (MB = 1 or 2 blocks
// of 128 rows sharing every dequantised weight tile, one TMEM accumulator of
// 256 columns each) over a K range.  Split-K (only when the tile grid cannot
// fill the SMs) launches the K ranges of a tile as one thread-block cluster and
// reduces the partial tiles through distributed shared memory.  Warp roles:
//   warp 0      weight producer: per 64-deep K stage, TMA of the packed weight
//               tile [64 x 32 words] and the stage's scale / zero rows into a
//               ring whose slots free as soon as they are dequantised;
//   warp 2      activation producer: TMA of the x tile [128 x 64] (K-major,
//               128B swizzle) into a ring whose slots free when the MMAs
//               reading them complete;
//   warp 1      owns the TMEM accumulators and issues, from one thread,
//               4 x MB tcgen05.mma (M128 N256 K16) per stage;
//   warps 3..   dequantise: each converts its packed words of a stage to
//               fp16/bf16 and stores them as the MN-major, 128B-swizzled B
//               operand of the MMA; after the last stage they drain TMEM
//               (tcgen05.ld) into y.
// Nibble pairs are unpacked with one LOP3 each (magic-exponent int4 -> fp16),
// which yields columns (0,4), (1,5), (2,6), (3,7) of a word; the B operand is
// stored in that column order and the epilogue undoes the permutation in
// registers.
#include <algorithm>

#include "w4a16_dq.cuh"

namespace b200q {
namespace tc {

// Grouped (per-expert) operation: blockIdx.y enumerates the 256-row tiles of
// every expert's contiguous row block [offsets[e], offsets[e+1]) of x (the
// routing kernel's grouping), expert e's weights are rows [e*K, (e+1)*K) of
// the stacked qweight (scales / zeros rows [e*K/g, (e+1)*K/g)).  With GLU the
// tile's 256 B-columns are 128 columns of the gate weight (tm_wq / tm_s /
// tm_z) and the same 128 columns of the up weight (wq2 / s2 / z2), and the
// epilogue writes h = SiLU(x.Wg) * (x.Wu) for those 128 columns.
struct Grouped {
  CUtensorMap wq2, s2, z2;
  const int32_t* offsets;
  int E;
};

enum { MODE_PLAIN = 0, MODE_GROUPED = 1, MODE_GLU = 2 };

template <bool BF16, int MB, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wq,
                    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                    const __grid_constant__ OutSet out, int M, int N, int K, int group, int splits, uint8_t* __restrict__ ws,
                    const __grid_constant__ Grouped grp) {
  constexpr bool GLU = MODE == MODE_GLU;
  constexpr int OUTC = GLU ? BN / 2 : BN;  // output columns per tile
  using T = typename DT<BF16>::T;
  using C = Cfg<MB>;
  constexpr int SX = C::SX, SW = C::SW, S2 = C::S2;
  constexpr uint32_t X_BYTES = C::X_BYTES, OFF_X = C::OFF_X, OFF_B = C::OFF_B, OFF_WQ = C::OFF_WQ,
                     OFF_S = C::OFF_S, OFF_Z = C::OFF_Z, OFF_BAR = C::OFF_BAR;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* x_full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* x_empty = x_full + SX;
  uint64_t* w_full = x_empty + SX;
  uint64_t* w_empty = w_full + SW;
  uint64_t* b_full = w_empty + SW;
  uint64_t* b_empty = b_full + S2;
  uint64_t* acc_full = b_empty + S2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ int s_err, s_clu_err;

  int* status = reinterpret_cast<int*>(ws);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z;
  const int n0 = n_tile * OUTC;  // first output (and weight) column of the tile
  int m0 = m_tile * BM * MB, m_end = M, wk0 = 0;
  int mb_act = MB;  // 128-row blocks of the tile that hold rows (grouped: an expert's last tile may need one)
  if (MODE != MODE_PLAIN) {
    // find this CTA's expert and row tile; CTAs past the last tile exit
    int e = 0, t = m_tile;
    for (; e < grp.E; ++e) {
      const int a = grp.offsets[e], b = grp.offsets[e + 1];
      const int tiles = (b - a + BM * MB - 1) / (BM * MB);
      if (t < tiles) {
        m0 = a + t * BM * MB;
        m_end = b;
        break;
      }
      t -= tiles;
    }
    if (e == grp.E) return;
    wk0 = e * K;
    mb_act = min(MB, (m_end - m0 + BM - 1) / BM);
  }
  const int nk_total = (K + BK - 1) / BK;
  const int k_begin = (int)((long long)split * nk_total / splits);
  const int k_end = (int)((long long)(split + 1) * nk_total / splits);
  const int nk = k_end - k_begin;
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
    fence_barrier_init();
    s_err = 0;
  }
  if (warp == W_PROD && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_wq);
    prefetch_tmap(&tm_s);
    prefetch_tmap(&tm_z);
  }
  if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) peer_arrive(out);
  if (warp == W_MMA) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == W_PROD) {
    // ---------------------------------------------------------------- weight producer
    if (lane == 0) {
      const uint32_t stage_tx = WQ_BYTES + 2u * srows * BN * 2u;
      for (int it = 0; it < nk; ++it) {
        const int s = it % SW;
        if (it >= SW && !mbar_wait(&w_empty[s], ((it / SW) - 1) & 1, status)) {
          s_err = 1;
          break;
        }
        const int kb = wk0 + (k_begin + it) * BK;
        mbar_arrive_expect_tx(&w_full[s], stage_tx);
        if (!GLU) {
          tma_load_2d(smem + OFF_WQ + s * WQ_BYTES, &tm_wq, n0 / 8, kb, &w_full[s]);
          tma_load_2d(smem + OFF_S + s * SZ_BYTES, &tm_s, n0, kb / group, &w_full[s]);
          tma_load_2d(smem + OFF_Z + s * SZ_BYTES, &tm_z, n0, kb / group, &w_full[s]);
        } else {
          // gate words then up words, [BK][16] each; scale / zero rows as
          // 128 gate columns then 128 up columns
          tma_load_2d(smem + OFF_WQ + s * WQ_BYTES, &tm_wq, n0 / 8, kb, &w_full[s]);
          tma_load_2d(smem + OFF_WQ + s * WQ_BYTES + WQ_BYTES / 2, &grp.wq2, n0 / 8, kb, &w_full[s]);
          for (int r = 0; r < srows; ++r) {
            uint8_t* srow = smem + OFF_S + s * SZ_BYTES + r * BN * 2;
            uint8_t* zrow = smem + OFF_Z + s * SZ_BYTES + r * BN * 2;
            tma_load_2d(srow, &tm_s, n0, kb / group + r, &w_full[s]);
            tma_load_2d(srow + BN, &grp.s2, n0, kb / group + r, &w_full[s]);
            tma_load_2d(zrow, &tm_z, n0, kb / group + r, &w_full[s]);
            tma_load_2d(zrow + BN, &grp.z2, n0, kb / group + r, &w_full[s]);
          }
        }
      }
    }
  } else if (warp == W_XPROD) {
    // ---------------------------------------------------------------- activation producer
    if (lane == 0) {
      for (int it = 0; it < nk; ++it) {
        const int s = it % SX;
        if (it >= SX && !mbar_wait(&x_empty[s], ((it / SX) - 1) & 1, status)) {
          s_err = 1;
          break;
        }
        const int kb = (k_begin + it) * BK;
        mbar_arrive_expect_tx(&x_full[s], mb_act * XB_BYTES);
#pragma unroll
        for (int mb = 0; mb < MB; ++mb)
          if (mb < mb_act)
            tma_load_2d(smem + OFF_X + s * X_BYTES + mb * XB_BYTES, &tm_x, kb, m0 + mb * BM, &x_full[s]);
      }
    }
  } else if (warp == W_MMA) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BM, BN, BF16 ? 1 : 0, /*a_mn=*/0, /*b_mn=*/1);
      for (int it = 0; it < nk; ++it) {
        const int s = it % SX, j = it % S2;
        if (!mbar_wait(&x_full[s], (it / SX) & 1, status) || !mbar_wait(&b_full[j], (it / S2) & 1, status)) {
          s_err = 1;
          break;
        }
        tc_fence_after();
        const uint32_t xa = smem_u32(smem + OFF_X + s * X_BYTES);
        const uint32_t bb = smem_u32(smem + OFF_B + j * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // A: K-major, 8-row groups 1024 B apart; B: MN-major, 64-column atoms
          // 1024 B apart, 8-row K groups 4096 B apart
          const uint64_t bd = smem_desc(bb + kk * 8192, 1024, 4096, 2);
#pragma unroll
          for (int mb = 0; mb < MB; ++mb) {
            if (mb >= mb_act) break;
            const uint64_t ad = smem_desc(xa + mb * XB_BYTES + kk * 32, 16, 1024, 2);
            tc_mma_f16_ss(tmem + mb * BN, ad, bd, idesc, (it | kk) != 0);
          }
        }
        tc_commit(&x_empty[s]);
        tc_commit(&b_empty[j]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ---------------------------------------------------------------- dequantise
    const int dw = warp - W_DQ0;
    const int nb = lane >> 3, ch = lane & 7;
    const int rr = dw & 7;  // row within each 8-row group
    static_assert(WPR == 2, "a thread's words i < WORDS/2 lie in K rows 0..31 of the stage, the rest in 32..63");
    // loop-invariant parts of every address; ring slots and phases advance
    // incrementally (no divisions in the loop)
    const uint32_t* wq_t = reinterpret_cast<const uint32_t*>(smem + OFF_WQ) +
                           (GLU ? (lane >> 4) * (BK * 16) + (rr + 8 * (dw >> 3)) * 16 + (lane & 15)
                                : (rr + 8 * (dw >> 3)) * 32 + lane);
    constexpr int WQ_ROW_STEP = GLU ? 8 * WPR * 16 : 8 * WPR * 32;  // words between a thread's words i, i+1
    uint8_t* b_t = smem + OFF_B + ((dw >> 3) * 4 + nb) * 1024 + rr * 128 + ((ch ^ rr) << 4);
    int s = 0, j = 0;
    uint32_t ph_w = 0, ph_b = 1;
    for (int it = 0; it < nk; ++it) {
      if (!mbar_wait(&w_full[s], ph_w, status)) {
        s_err = 1;
        break;
      }
      if (it >= S2 && !mbar_wait(&b_empty[j], ph_b, status)) {
        s_err = 1;
        break;
      }
      const uint8_t* srow0 = smem + OFF_S + s * SZ_BYTES;
      const uint8_t* zrow0 = smem + OFF_Z + s * SZ_BYTES;
      // packed words and scale/zero constants go to registers first, so the
      // weight slot is released before the dequantised stores start; with
      // group 32 the stage's second scale row serves K rows 32..63 (words
      // i >= WORDS/2), otherwise q1 is q0
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
      if (++s == SW) {
        s = 0;
        ph_w ^= 1;
      }
      if (++j == S2) {
        j = 0;
        ph_b ^= 1;
      }
    }

    // ---------------------------------------------------------------- epilogue: TMEM -> y
    // The tile is staged in shared memory (the operand rings are idle once the
    // accumulator is complete) as rows of OUTC output values: CH 16-byte
    // chunks per row, the chunk index XOR-swizzled by the row so that both the
    // row-per-lane writes here and the chunk-per-lane reads below are free of
    // bank conflicts.  Rows then leave as whole lines (512 B, or 256 B with
    // GLU), coalesced in HBM and as few, large NVLink writes.
    constexpr int CH = OUTC / 8;
    const bool acc_ok = !s_err && mbar_wait(acc_full, 0, status);
    if (!acc_ok) s_err = 1;
    if (acc_ok) {
      tc_fence_after();
      const int qd = warp & 3;   // TMEM lane quadrant this warp may access
      const int part = dw >> 2;  // which of the NDQ/4 column ranges of this quadrant
      constexpr int COLS = MB * OUTC / (NDQ / 4);  // lies within one accumulator
      const int acc = (part * COLS) / OUTC;
      const int trow = acc * BM + qd * 32 + lane;  // row within the CTA tile
      const uint32_t tl = tmem + ((uint32_t)(qd * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < COLS; c0 += 32) {
        const int tcol = part * COLS + c0;  // output column tcol % OUTC of accumulator acc
        const int ocol = tcol % OUTC;
        uint32_t r[32];
        float v[32];
        tmem_ld32(tl + acc * BN + ocol, r);
        tmem_ld_wait();
#pragma unroll
        for (int p = 0; p < 32; ++p) v[(p & ~7) | slot_col(p & 7)] = __uint_as_float(r[p]);
        if (GLU) {
          // up columns sit 128 TMEM columns to the right; h = SiLU(g) * u with
          // g and u rounded to the activation type first and one rounding of
          // the product, as the unfused gate/up GEMMs + silu_mul compute it
          tmem_ld32(tl + acc * BN + ocol + BN / 2, r);
          tmem_ld_wait();
#pragma unroll
          for (int p = 0; p < 32; ++p) {
            const float g = (float)(T)v[(p & ~7) | slot_col(p & 7)];
            const float u = (float)(T)__uint_as_float(r[p]);
            v[(p & ~7) | slot_col(p & 7)] = g / (1.f + expf(-g)) * u;
          }
        }
        if (splits == 1) {
          uint32_t packed[16];
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            if (!BF16)
              packed[p] = as_u32(__floats2half2_rn(v[2 * p], v[2 * p + 1]));
            else
              packed[p] = as_u32(__floats2bfloat162_rn(v[2 * p], v[2 * p + 1]));
          }
          uint8_t* srow = smem + (uint32_t)trow * (OUTC * 2);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int chunk = (ocol >> 3) + p;
            *reinterpret_cast<uint4*>(srow + ((chunk ^ (trow % CH)) << 4)) =
                make_uint4(packed[4 * p], packed[4 * p + 1], packed[4 * p + 2], packed[4 * p + 3]);
          }
        }
      }
    }
    if (splits == 1) {
      if (warp == W_DQ0 && lane == 0 && !s_err && !peer_wait_arrivals(out, status)) s_err = 1;
      named_barrier_sync(1, NDQ * 32);  // all epilogue warps, failed or not
      if (!s_err) {
        constexpr int RPW = 32 / CH;  // rows per warp instruction
        const int chunk = lane % CH;
        const int col = n0 + chunk * 8;
#pragma unroll 1
        for (int r = dw * RPW + lane / CH; r < MB * BM; r += NDQ * RPW) {
          const int grow = m0 + r;
          if (grow >= m_end) break;
          const uint4 val =
              *reinterpret_cast<const uint4*>(smem + (uint32_t)r * (OUTC * 2) + ((chunk ^ (r % CH)) << 4));
          if (col < N)
            for (int o = 0; o < out.n; ++o)
              *reinterpret_cast<uint4*>(reinterpret_cast<T*>(out.y[o]) + (size_t)grow * out.ldy + out.col0 + col) =
                  val;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (splits > 1) {
    // split-K across the CTAs of this cluster (one per K range): rows
    // [lo(o), lo(o + 1)) of the tile, lo(o) = o * BM / S, are owned by cluster
    // rank o (S any of 2..8, so the row blocks may differ by one row).  Each
    // CTA sends its partial rows to the owners' shared memory (the pipeline
    // buffers, free once every CTA passed the first cluster barrier) at
    // [sender rank][row - lo(owner)], MAXR rows per sender; then every owner
    // sums the S partials in rank order and writes y: the result does not
    // depend on timing, and no global workspace is used.  A 256-row tile
    // (MB = 2) is reduced in two passes of one 128-row block each, so the
    // received partials never exceed S * MAXR rows of fp32.
    const uint32_t S = (uint32_t)splits, MAXR = (BM + S - 1) / S;
    const uint32_t rank = cluster_ctarank();
    for (int mb = 0; mb < MB; ++mb) {
    cluster_sync();  // every CTA is done with its pipeline buffers / the previous pass
    if (warp >= W_DQ0 && !s_err) {
      tc_fence_after();
      const int dw = warp - W_DQ0;
      const int qd = warp & 3, part = dw >> 2;
      constexpr int COLS = BN / (NDQ / 4);
      const uint32_t trow = qd * 32 + lane;
      uint32_t owner = trow * S / BM;
      while ((owner + 1) * BM / S <= trow) ++owner;
      const uint32_t lr = trow - owner * BM / S;
      const uint32_t base = map_shared_rank(smem_u32(smem), owner) + ((rank * MAXR + lr) * BN) * 4;
#pragma unroll 1
      for (int c0 = 0; c0 < COLS; c0 += 32) {
        const int cslot = part * COLS + c0;
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(qd * 32) << 16) + mb * BN + cslot, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int p = 0; p < 32; ++p) v[(p & ~7) | slot_col(p & 7)] = __uint_as_float(r[p]);
#pragma unroll
        for (int p = 0; p < 8; ++p)
          st_cluster_v4(base + (cslot + 4 * p) * 4, v[4 * p], v[4 * p + 1], v[4 * p + 2], v[4 * p + 3]);
      }
    }
    if (mb == 0 && threadIdx.x == 0 && !s_err && !peer_wait_arrivals(out, status)) s_err = 1;
    cluster_sync();
    // a CTA of the cluster that gave up a wait sent incomplete rows: then no
    // owner of the cluster writes this pass (every CTA's s_err is final here)
    if (threadIdx.x == 0) s_clu_err = 0;
    __syncthreads();
    if (threadIdx.x < S) {
      int e;
      asm volatile("ld.shared::cluster.s32 %0, [%1];"
                   : "=r"(e)
                   : "r"(map_shared_rank(smem_u32(&s_err), threadIdx.x)));
      if (e) atomicOr(&s_clu_err, 1);
    }
    __syncthreads();
    if (!s_clu_err) {
      const float* buf = reinterpret_cast<const float*>(smem);
      const int r0 = (int)(rank * BM / S), nr = (int)((rank + 1) * BM / S) - r0;
      for (int e = threadIdx.x * 4; e < nr * BN; e += THREADS * 4) {
        const int lr = e / BN, c = e % BN;
        float4 acc4 = reinterpret_cast<const float4*>(buf + lr * BN + c)[0];
        for (uint32_t src = 1; src < S; ++src) {
          const float4 p4 = reinterpret_cast<const float4*>(buf + (src * MAXR + lr) * BN + c)[0];
          acc4.x += p4.x;
          acc4.y += p4.y;
          acc4.z += p4.z;
          acc4.w += p4.w;
        }
        const int row = m0 + mb * BM + r0 + lr, col = n0 + c;
        if (row < m_end && col < N) {
          uint2 packed;
          if (!BF16) {
            packed.x = as_u32(__floats2half2_rn(acc4.x, acc4.y));
            packed.y = as_u32(__floats2half2_rn(acc4.z, acc4.w));
          } else {
            packed.x = as_u32(__floats2bfloat162_rn(acc4.x, acc4.y));
            packed.y = as_u32(__floats2bfloat162_rn(acc4.z, acc4.w));
          }
          for (int o = 0; o < out.n; ++o)
            *reinterpret_cast<uint2*>(reinterpret_cast<T*>(out.y[o]) + (size_t)row * out.ldy + out.col0 + col) =
                packed;
        }
      }
    }
    }  // passes over the 128-row blocks
  }
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
  int mb, tiles_m, tiles_n, splits;
  size_t ws_bytes;
};

Plan plan(int64_t M, int64_t N, int64_t K, int sms) {
  Plan p;
  p.tiles_n = (int)((N + BN - 1) / BN);
  const int nk = (int)((K + BK - 1) / BK);
  // split-K: the K ranges of a tile form one thread-block cluster (at most 8,
  // the portable cluster size), as many as the SMs allow, keeping >= 4
  // stages per range; the launch shrinks it further until every cluster of
  // the grid is co-resident
  auto split_for = [&](int64_t tiles) {
    int64_t sp = sms / tiles;
    if (sp > nk / 4) sp = nk / 4;
    if (sp > MAX_SPLITS) sp = MAX_SPLITS;
    return (int)(sp < 1 ? 1 : sp);
  };
  // estimated time in 128-row stage-times: waves of tiles x splits CTAs,
  // each running nk / splits stages; a 256-row tile halves the
  // dequantisation per FLOP but its stage costs ~1.35x a 128-row one (measured)
  auto cost = [&](int64_t tiles, int sp, double stage) {
    const int64_t waves = (tiles * sp + sms - 1) / sms;
    return stage * (double)waves * (double)((nk + sp - 1) / sp);
  };
  const int64_t tiles1 = ((M + BM - 1) / BM) * p.tiles_n;
  const int64_t tiles2 = ((M + 2 * BM - 1) / (2 * BM)) * p.tiles_n;
  const int sp1 = split_for(tiles1), sp2 = split_for(tiles2);
  // (up to M = 256 the 128-row split with one DSMEM pass measured faster
  // than the 256-row split reduced in two passes: 48.8 vs 51.9 us at M = 256)
  p.mb = (M > 2 * BM && cost(tiles2, sp2, 1.35) < cost(tiles1, sp1, 1.0)) ? 2 : 1;
  p.tiles_m = (int)((M + BM * p.mb - 1) / (BM * p.mb));
  p.splits = p.mb == 2 ? sp2 : sp1;
  p.ws_bytes = HEADER_BYTES;
  return p;
}

}  // namespace tc

size_t w4a16_tc_ws_bytes(int64_t M, int64_t N, int64_t K, int device) {
  return tc::plan(M, N, K, num_sms(device)).ws_bytes;
}

int w4a16_tc(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& out,
             int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace, size_t workspace_bytes,
             cudaStream_t stream) {
  using namespace tc;
  Plan p = plan(M, N, K, num_sms(-1));
  if (!workspace || workspace_bytes < p.ws_bytes)
    return fail(B200Q_ERR_WORKSPACE, "w4a16: workspace of " + std::to_string(p.ws_bytes) + " bytes required");
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
  auto kern = p.mb == 2 ? (bf ? w4a16_tc_kernel<true, 2, MODE_PLAIN> : w4a16_tc_kernel<false, 2, MODE_PLAIN>)
                        : (bf ? w4a16_tc_kernel<true, 1, MODE_PLAIN> : w4a16_tc_kernel<false, 1, MODE_PLAIN>);
  const uint32_t smem = p.mb == 2 ? Cfg<2>::SMEM : Cfg<1>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(w4a16 tc)");
  // a cluster of `splits` CTAs (one SM each) must fit in one GPC: shrink the
  // cluster until every cluster of the grid is resident at once
  while (p.splits > 1) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(p.tiles_n, p.tiles_m, p.splits);
    q.blockDim = dim3(THREADS);
    q.dynamicSmemBytes = smem;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 1;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = (unsigned)p.splits;
    q.attrs = qa;
    q.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, kern, &q) == cudaSuccess && active >= p.tiles_m * p.tiles_n) break;
    cudaGetLastError();
    --p.splits;
  }
  dim3 grid(p.tiles_n, p.tiles_m, p.splits);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)p.splits;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Grouped none = {};
  e = cudaLaunchKernelEx(&cfg, kern, tx, twq, ts, tz, out, (int)M, (int)N, (int)K, (int)group, p.splits,
                         reinterpret_cast<uint8_t*>(workspace), none);
  if (e != cudaSuccess) return check_cuda(e, "w4a16 tc launch");
  return check_cuda(cudaGetLastError(), "w4a16 tc launch");
}

// Grouped W4A16 over E experts (the MoE expert GEMMs in one launch): rows of
// x [rows, K] are grouped by expert, offsets [E + 1] on the device; weights are
// stacked per expert (qweight [E*K, N/8], scales / zeros [E*K/g, N]).  With
// glu, N is the hidden width, the second weight set is the up projection and
// y [rows, N] = SiLU(x.Wg) * (x.Wu); without, y = x.W.
int w4a16_tc_grouped(const void* x, const int32_t* qw, const void* sc, const void* zr, const int32_t* qw2,
                     const void* sc2, const void* zr2, const int32_t* offsets, int64_t E, void* y, int64_t rows,
                     int64_t N, int64_t K, int64_t group, int dtype, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream) {
  using namespace tc;
  const bool glu = qw2 != nullptr;
  if (!workspace || workspace_bytes < (size_t)HEADER_BYTES)
    return fail(B200Q_ERR_WORKSPACE, "w4a16 grouped: workspace of " + std::to_string(HEADER_BYTES) + " bytes required");
  if (rows == 0) return B200Q_OK;
  const CUtensorMapDataType h16 = CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const uint32_t wbox = glu ? BN / 16 : BN / 8, cbox = glu ? BN / 2 : BN;
  const uint32_t srows = glu ? 1 : (group >= BK ? 1 : (uint32_t)(BK / group));
  const uint64_t krows = (uint64_t)E * K, grows = (uint64_t)E * (K / group);
  CUtensorMap tx, twq, ts, tz;
  Grouped g = {};
  int rc;
  if ((rc = encode_2d(&tx, h16, x, K, rows, (uint64_t)K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  auto enc_w = [&](CUtensorMap* wm, CUtensorMap* sm, CUtensorMap* zm, const int32_t* q, const void* s_,
                   const void* z_) -> int {
    int r;
    if ((r = encode_2d(wm, CU_TENSOR_MAP_DATA_TYPE_INT32, q, N / 8, krows, (uint64_t)N / 2, wbox, BK,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
      return r;
    if ((r = encode_2d(sm, h16, s_, N, grows, (uint64_t)N * 2, cbox, srows, CU_TENSOR_MAP_SWIZZLE_NONE))) return r;
    return encode_2d(zm, h16, z_, N, grows, (uint64_t)N * 2, cbox, srows, CU_TENSOR_MAP_SWIZZLE_NONE);
  };
  if ((rc = enc_w(&twq, &ts, &tz, qw, sc, zr))) return rc;
  if (glu && (rc = enc_w(&g.wq2, &g.s2, &g.z2, qw2, sc2, zr2))) return rc;
  g.offsets = offsets;
  g.E = (int)E;
  const bool bf = dtype == B200Q_DTYPE_BF16;
  // 256-row tiles: one dequantised weight tile serves up to 256 of an
  // expert's rows (the second 128-row block is skipped when the tile has no
  // more than 128 rows)
  auto kern = glu ? (bf ? w4a16_tc_kernel<true, 2, MODE_GLU> : w4a16_tc_kernel<false, 2, MODE_GLU>)
                  : (bf ? w4a16_tc_kernel<true, 2, MODE_GROUPED> : w4a16_tc_kernel<false, 2, MODE_GROUPED>);
  const uint32_t smem = Cfg<2>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(w4a16 grouped)");
  // every expert's rows in 256-row tiles: at most rows/256 + E tiles
  const int tiles_m = (int)((rows + 2 * BM - 1) / (2 * BM) + E);
  const int tiles_n = (int)((N + (glu ? BN / 2 : BN) - 1) / (glu ? BN / 2 : BN));
  OutSet out = single_out(y, N);
  // split-K (plain grouped mode): when the experts' tiles cannot fill the
  // SMs (expert-parallel ranks hold few rows per expert), the K ranges of a
  // tile form a cluster, as in the dense kernel.  The tile count is only known
  // on the device; the estimate is one 256-row tile per expert or per 256
  // rows, whichever is more (tiles launched beyond the real ones exit at once).
  int splits = 1;
  if (!glu) {
    const int nk = (int)((K + BK - 1) / BK);
    const int est_m = (int)std::min<int64_t>(tiles_m, std::max<int64_t>(E, (rows + 2 * BM - 1) / (2 * BM)));
    const int sms = num_sms(-1);
    splits = sms / std::max(1, est_m * tiles_n);
    splits = std::max(1, std::min(splits, std::min(MAX_SPLITS, nk / 4)));
    while (splits > 1) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(tiles_n, est_m, splits);
      q.blockDim = dim3(THREADS);
      q.dynamicSmemBytes = smem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 1;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = (unsigned)splits;
      q.attrs = qa;
      q.numAttrs = 1;
      int active = 0;
      if (cudaOccupancyMaxActiveClusters(&active, kern, &q) == cudaSuccess && active >= est_m * tiles_n) break;
      cudaGetLastError();
      --splits;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles_n, tiles_m, splits);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)splits;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tx, twq, ts, tz, out, (int)rows, (int)N, (int)K, (int)group, splits,
                         reinterpret_cast<uint8_t*>(workspace), g);
  if (e != cudaSuccess) return check_cuda(e, "w4a16 grouped launch");
  return check_cuda(cudaGetLastError(), "w4a16 grouped launch");
}

}  // namespace b200q
