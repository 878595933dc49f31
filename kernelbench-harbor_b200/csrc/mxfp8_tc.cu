// MXFP8 block-scaled GEMM on the tcgen05 tensor cores
// (kind::mxf8f6f4.block_scale): y[M, N] = fp16( A_deq . B_deq^T ), A [M, K] and
// B [N, K] e4m3 (both K-major), one E8M0 scale per 32 consecutive K elements
// of each row (scales_a [M, K/32], scales_b [N, K/32], bias 127), fp32
// accumulation in tensor memory.  The reference's closest module is FP8_REF
// (generate_tasks.py:218-237, weight-only fp8 with fp16 block scales); the MX
// configuration follows the OCP Microscaling v1.0 format.
//
// One CTA: a 128 x 256 output tile over a K range.  When the tiles cannot fill
// the SMs, the K ranges of a tile form one thread-block cluster (split-K): each
// CTA sends its accumulator rows to the owning CTA's shared memory over DSMEM
// and the owners sum them in rank order (deterministic, no workspace).  The
// epilogue stores each finished tile into every destination of an OutSet, so
// the column-sharded multi-GPU GEMM's all-gather is fused into it (NVLink peer
// stores of whole 512-byte rows, ordered through the signal pads as in the
// W4A16 kernels).  Warp 0: TMA producer (A box [128 x 128 k],
// B box [256 x 128 k], 4-deep ring); warp 1: TMEM owner and MMA issuer (4 x
// M128 N256 K32 per 128-deep stage); warps 2..5: per stage they load the
// stage's scale factors (one 32-bit word = 4 K-blocks per row) and write them
// into tensor memory with tcgen05.st, laid out as the block-scaled MMA reads
// them: for a matrix of R rows, row r's scale in byte 0 of column C + r/32,
// lane r%32, replicated in the four lane quadrants, with its own columns for
// each MMA (K-block); they also drain the accumulator in the epilogue.
#include "common.cuh"

namespace b200q {
namespace mx {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int THREADS = 6 * 32;
constexpr uint32_t A_BYTES = BM * BK;  // 16 KB
constexpr uint32_t B_BYTES = BN * BK;  // 32 KB
constexpr uint32_t STAGE = A_BYTES + B_BYTES;
constexpr uint32_t OFF_BAR = STAGES * STAGE;
constexpr uint32_t SMEM = OFF_BAR + 256 + 1024;
constexpr int SF_COL0 = 256;      // TMEM columns of the scale factors (after the accumulator)
constexpr int SF_MMA = 12;        // per MMA: SFA 4 columns, SFB 8 columns (scale in byte 0)
constexpr int SF_STRIDE = 4 * SF_MMA;  // per ring slot (4 MMAs per stage)
constexpr int HEADER_BYTES = 256;
constexpr int MAX_SPLITS = 8;  // portable cluster size
static_assert(SMEM <= 227 * 1024, "shared memory budget");

__global__ void __launch_bounds__(THREADS, 1)
    mxfp8_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const uint32_t* __restrict__ sfa, const uint32_t* __restrict__ sfb,
                    const __grid_constant__ OutSet out, int M, int N, int K, int splits, int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* sf_full = empty + STAGES;
  uint64_t* sf_empty = sf_full + STAGES;
  uint64_t* acc_full = sf_empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ int s_err, s_any_err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z;
  const int n0 = n_tile * BN, m0 = m_tile * BM;
  const int nk_total = K / BK;
  const int k_begin = (int)((long long)split * nk_total / splits);
  const int nk = (int)((long long)(split + 1) * nk_total / splits) - k_begin;
  const int kw = K / 128;  // 32-bit scale words per row (4 K-blocks each)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_full[s], 4);
      mbar_init(&sf_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
    s_err = 0;
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) peer_arrive(out);
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int it = 0; it < nk; ++it) {
        const int s = it % STAGES;
        if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, status)) {
          s_err = 1;
          break;
        }
        const int kb = (k_begin + it) * BK;
        uint8_t* st = smem + s * STAGE;
        mbar_arrive_expect_tx(&full[s], STAGE);
        tma_load_2d(st, &tm_a, kb, m0, &full[s]);
        tma_load_2d(st + A_BYTES, &tm_b, kb, n0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int it = 0; it < nk; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, status) || !mbar_wait(&sf_full[s], (it / STAGES) & 1, status)) {
          s_err = 1;
          break;
        }
        tc_fence_after();
        const uint32_t aa = smem_u32(smem + s * STAGE);
        const uint32_t ba = aa + A_BYTES;
        const uint32_t idesc = idesc_mxf8(BM, BN, 0, 0);
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk) {
          // both operands K-major, 128B swizzle: 32 e4m3 = 32 B per K step
          const uint64_t ad = smem_desc(aa + kk * 32, 16, 1024, 2);
          const uint64_t bd = smem_desc(ba + kk * 32, 16, 1024, 2);
          const uint32_t sf = tmem + SF_COL0 + s * SF_STRIDE + kk * SF_MMA;
          tc_mma_mxf8_ss(tmem, ad, bd, idesc, sf, sf + 4, (it | kk) != 0);
        }
        tc_commit(&empty[s]);
        tc_commit(&sf_empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ---------------------------------------------------------------- scale factors -> TMEM (warps 2..5)
    const int qd = warp & 3;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    // Scale words are prefetched SF_AHEAD stages ahead in registers: their
    // global loads do not depend on the TMEM slot being free, only the stores do.
    constexpr int SF_AHEAD = 3;
    uint32_t pre[SF_AHEAD][12];
    auto load_sf = [&](int it, uint32_t* w) {
      const int wcol = k_begin + it;  // scale word column: K-blocks 4*wcol .. 4*wcol+3
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = m0 + 32 * j + lane;
        w[j] = (it < nk && r < M) ? __ldg(sfa + (size_t)r * kw + wcol) : 0u;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = n0 + 32 * j + lane;
        w[4 + j] = (it < nk && r < N) ? __ldg(sfb + (size_t)r * kw + wcol) : 0u;
      }
    };
#pragma unroll
    for (int d = 0; d < SF_AHEAD; ++d) load_sf(d, pre[d]);
    for (int it = 0; it < nk; ++it) {
      const int s = it % STAGES;
      uint32_t cur[12];
#pragma unroll
      for (int i = 0; i < 12; ++i) cur[i] = pre[0][i];
#pragma unroll
      for (int d = 0; d + 1 < SF_AHEAD; ++d)
#pragma unroll
        for (int i = 0; i < 12; ++i) pre[d][i] = pre[d + 1][i];
      load_sf(it + SF_AHEAD, pre[SF_AHEAD - 1]);
      if (it >= STAGES && !mbar_wait(&sf_empty[s], ((it / STAGES) - 1) & 1, status)) {
        s_err = 1;
        break;
      }
      // one K-block per MMA: byte kk of each row's word goes to byte 0 of that
      // MMA's scale columns
#pragma unroll
      for (int kk = 0; kk < BK / 32; ++kk) {
        uint32_t ka[4], kb_[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) ka[j] = (cur[j] >> (8 * kk)) & 0xFFu;
#pragma unroll
        for (int j = 0; j < 8; ++j) kb_[j] = (cur[4 + j] >> (8 * kk)) & 0xFFu;
        const uint32_t sf = tmem + SF_COL0 + s * SF_STRIDE + kk * SF_MMA;
        tmem_st4(sf + lane_base, ka);
        tmem_st8(sf + 4 + lane_base, kb_);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sf_full[s]);
    }
    // ---------------------------------------------------------------- epilogue (no split)
    // the tile is staged in shared memory as fp16 (the ring is idle once the
    // accumulator is complete), 16-byte chunks XOR-swizzled by row, and then
    // leaves as whole rows
    if (splits == 1 && !s_err && mbar_wait(acc_full, 0, status)) {
      tc_fence_after();
      const int trow = qd * 32 + lane;
      uint8_t* srow = smem + (uint32_t)trow * (BN * 2);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + c0, r);
        tmem_ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          __half2 h = __floats2half2_rn(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1]));
          packed[p] = *reinterpret_cast<uint32_t*>(&h);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int chunk = (c0 >> 3) + p;
          *reinterpret_cast<uint4*>(srow + ((chunk ^ (trow & 31)) << 4)) =
              make_uint4(packed[4 * p], packed[4 * p + 1], packed[4 * p + 2], packed[4 * p + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (splits == 1) {
    if (threadIdx.x == 0 && !s_err && !peer_wait_arrivals(out, status)) s_err = 1;
    __syncthreads();
    if (!s_err) {
      const int rows = min(BM, M - m0);
      for (int e = threadIdx.x; e < rows * (BN / 8); e += THREADS) {
        const int r = e / (BN / 8), chunk = e % (BN / 8);
        const int col = n0 + chunk * 8;
        if (col >= N) continue;  // N % 32 == 0: a chunk is wholly inside or outside
        const uint4 v = *reinterpret_cast<const uint4*>(smem + (uint32_t)r * (BN * 2) + ((chunk ^ (r & 31)) << 4));
        for (int o = 0; o < out.n; ++o)
          *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out.y[o]) + (size_t)(m0 + r) * out.ldy + out.col0 +
                                    col) = v;
      }
    }
  } else {
    // split-K across the CTAs of this cluster (one per K range): rows
    // [o * BM / S, (o + 1) * BM / S) of the tile belong to cluster rank o.
    // Every CTA sends its accumulator rows to the owners' shared memory at
    // [sender rank][row - first row of the owner] (MAXR rows per sender);
    // after a cluster barrier each owner sums the S partials in rank order.
    const uint32_t S = (uint32_t)splits, MAXR = (BM + S - 1) / S;
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) s_any_err = s_err;
    cluster_sync();  // every CTA is done with its ring (the receive buffer)
    if (warp >= 2 && !s_err && mbar_wait(acc_full, 0, status)) {
      tc_fence_after();
      const int qd = warp & 3;
      const uint32_t trow = qd * 32 + lane;
      uint32_t owner = trow * S / BM;
      while ((owner + 1) * BM / S <= trow) ++owner;
      const uint32_t lr = trow - owner * BM / S;
      const uint32_t base = map_shared_rank(smem_u32(smem), owner) + ((rank * MAXR + lr) * BN) * 4;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(qd * 32) << 16) + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int p = 0; p < 8; ++p)
          st_cluster_v4(base + (c0 + 4 * p) * 4, __uint_as_float(r[4 * p]), __uint_as_float(r[4 * p + 1]),
                        __uint_as_float(r[4 * p + 2]), __uint_as_float(r[4 * p + 3]));
      }
    }
    if (threadIdx.x == 0 && !s_err && !peer_wait_arrivals(out, status)) s_err = 1;
    cluster_sync();
    // a CTA that gave up a wait sent nothing: then no owner of the cluster stores
    if (threadIdx.x < splits) {
      int e;
      asm volatile("ld.shared::cluster.s32 %0, [%1];"
                   : "=r"(e)
                   : "r"(map_shared_rank(smem_u32(&s_any_err), (uint32_t)threadIdx.x)));
      if (e) atomicOr(&s_err, 1);
    }
    __syncthreads();
    if (!s_err) {
      const float* buf = reinterpret_cast<const float*>(smem);
      const int r0 = (int)(rank * BM / S), nr = (int)((rank + 1) * BM / S) - r0;
      for (int e = threadIdx.x * 8; e < nr * BN; e += THREADS * 8) {
        const int lr = e / BN, c = e % BN;
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = 0.f;
        for (uint32_t src = 0; src < S; ++src) {
          const float4 p0 = reinterpret_cast<const float4*>(buf + (src * MAXR + lr) * BN + c)[0];
          const float4 p1 = reinterpret_cast<const float4*>(buf + (src * MAXR + lr) * BN + c)[1];
          v[0] += p0.x, v[1] += p0.y, v[2] += p0.z, v[3] += p0.w;
          v[4] += p1.x, v[5] += p1.y, v[6] += p1.z, v[7] += p1.w;
        }
        const int row = m0 + r0 + lr, col = n0 + c;
        if (row < M && col < N) {
          uint32_t packed[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __half2 h = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
            packed[q] = *reinterpret_cast<uint32_t*>(&h);
          }
          const uint4 val = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          for (int o = 0; o < out.n; ++o)
            *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out.y[o]) + (size_t)row * out.ldy + out.col0 + col) =
                val;
        }
      }
    }
    cluster_sync();  // no CTA exits while its buffer may still be read
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (out.world > 1) {
    __syncthreads();
    if (threadIdx.x < 32) peer_finish(out, status);
  }
}

struct Plan {
  int tiles_m, tiles_n, splits;
};

Plan plan(int64_t M, int64_t N, int64_t K, int sms) {
  Plan p;
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)((N + BN - 1) / BN);
  const int nk = (int)(K / BK);
  int sp = sms / (p.tiles_m * p.tiles_n);
  if (sp < 1) sp = 1;
  if (sp > MAX_SPLITS) sp = MAX_SPLITS;
  if (sp > nk / 2) sp = nk / 2 > 0 ? nk / 2 : 1;
  p.splits = sp;
  return p;
}

}  // namespace mx

int mxfp8_tc(const void* a, const void* scales_a, const void* b, const void* scales_b, const OutSet& out, int64_t M,
             int64_t N, int64_t K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace mx;
  if (!workspace || workspace_bytes < (size_t)HEADER_BYTES)
    return fail(B200Q_ERR_WORKSPACE, "mxfp8: workspace of " + std::to_string(HEADER_BYTES) + " bytes required");
  Plan p = plan(M, N, K, num_sms(-1));
  CUtensorMap ta, tb;
  int rc;
  if ((rc = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, K, M, (uint64_t)K, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, K, N, (uint64_t)K, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  cudaError_t e = cudaFuncSetAttribute(mxfp8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(mxfp8)");
  // a cluster of `splits` CTAs (one SM each) must fit in one GPC: shrink the
  // cluster until every cluster of the grid is resident at once
  while (p.splits > 1) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(p.tiles_n, p.tiles_m, p.splits);
    q.blockDim = dim3(THREADS);
    q.dynamicSmemBytes = SMEM;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 1;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = (unsigned)p.splits;
    q.attrs = qa;
    q.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, mxfp8_tc_kernel, &q) == cudaSuccess &&
        active >= p.tiles_m * p.tiles_n)
      break;
    cudaGetLastError();
    --p.splits;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.tiles_n, p.tiles_m, p.splits);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)p.splits;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, mxfp8_tc_kernel, ta, tb, reinterpret_cast<const uint32_t*>(scales_a),
                         reinterpret_cast<const uint32_t*>(scales_b), out, (int)M, (int)N, (int)K, p.splits,
                         reinterpret_cast<int*>(workspace));
  if (e != cudaSuccess) return check_cuda(e, "mxfp8 launch");
  return check_cuda(cudaGetLastError(), "mxfp8 launch");
}

}  // namespace b200q

extern "C" {

size_t b200q_mxfp8_workspace_bytes(int64_t, int64_t, int64_t, int) { return b200q::mx::HEADER_BYTES; }

int b200q_mxfp8_gemm(const void* a, const void* scales_a, const void* b, const void* scales_b, void* y, int64_t M,
                     int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace b200q;
  if (M < 0 || N <= 0 || K <= 0) return fail(B200Q_ERR_SHAPE, "mxfp8: M must be >= 0 and N, K > 0");
  if (K % 128) return fail(B200Q_ERR_SHAPE, "mxfp8: K must be a multiple of 128");
  if (N % 32) return fail(B200Q_ERR_ALIGN, "mxfp8: N must be a multiple of 32");
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return fail(B200Q_ERR_SHAPE, "mxfp8: size too large");
  if (M == 0) return B200Q_OK;
  if (!a || !scales_a || !b || !scales_b || !y) return fail(B200Q_ERR_SHAPE, "mxfp8: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(scales_a) | reinterpret_cast<uintptr_t>(scales_b)) & 3)
    return fail(B200Q_ERR_ALIGN, "mxfp8: scale arrays must be 4-byte aligned");
  if (reinterpret_cast<uintptr_t>(y) & 15) return fail(B200Q_ERR_ALIGN, "mxfp8: y must be 16-byte aligned");
  return mxfp8_tc(a, scales_a, b, scales_b, single_out(y, N), M, N, K, workspace, workspace_bytes,
                  reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
