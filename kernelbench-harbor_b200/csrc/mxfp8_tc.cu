// MXFP8 block-scaled GEMM on the tcgen05 tensor cores
// (kind::mxf8f6f4.block_scale): y[M, N] = fp16( A_deq . B_deq^T ), A [M, K] and
// B [N, K] e4m3 (both K-major), one E8M0 scale per 32 consecutive K elements
// of each row (scales_a [M, K/32], scales_b [N, K/32], bias 127), fp32
// accumulation in tensor memory.  The reference's closest module is FP8_REF
// (generate_tasks.py:218-237, weight-only fp8 with fp16 block scales); the MX
// configuration follows the OCP Microscaling v1.0 format.
//
// One CTA: a 128 x 256 output tile over a K range (split-K with fp32 atomics
// when the tiles cannot fill the SMs).  Warp 0: TMA producer (A box [128 x 128 k],
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
constexpr int MAX_SPLITS = 16;
static_assert(SMEM <= 227 * 1024, "shared memory budget");

__global__ void __launch_bounds__(THREADS, 1)
    mxfp8_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const uint32_t* __restrict__ sfa, const uint32_t* __restrict__ sfb, __half* __restrict__ y,
                    int M, int N, int K, int splits, uint8_t* __restrict__ ws) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* sf_full = empty + STAGES;
  uint64_t* sf_empty = sf_full + STAGES;
  uint64_t* acc_full = sf_empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ int s_err, s_last;

  int* status = reinterpret_cast<int*>(ws);
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
    // ---------------------------------------------------------------- epilogue
    if (!s_err && mbar_wait(acc_full, 0, status)) {
      tc_fence_after();
      const int row = m0 + qd * 32 + lane;
      float* acc_ws = reinterpret_cast<float*>(ws + HEADER_BYTES);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + c0, r);
        tmem_ld_wait();
        const int col = n0 + c0;
        if (row >= M || col >= N) continue;
        if (splits == 1) {
          uint32_t packed[16];
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            __half2 h = __floats2half2_rn(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1]));
            packed[p] = *reinterpret_cast<uint32_t*>(&h);
          }
          uint4* dst = reinterpret_cast<uint4*>(y + (size_t)row * N + col);
#pragma unroll
          for (int p = 0; p < 4; ++p)
            dst[p] = make_uint4(packed[4 * p], packed[4 * p + 1], packed[4 * p + 2], packed[4 * p + 3]);
        } else {
          float4* dst = reinterpret_cast<float4*>(acc_ws + (size_t)row * N + col);
#pragma unroll
          for (int p = 0; p < 8; ++p)
            atomicAdd(dst + p, make_float4(__uint_as_float(r[4 * p]), __uint_as_float(r[4 * p + 1]),
                                           __uint_as_float(r[4 * p + 2]), __uint_as_float(r[4 * p + 3])));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (splits > 1 && !s_err) {
    __threadfence();
    __syncthreads();
    int* tickets = reinterpret_cast<int*>(ws + HEADER_BYTES + (size_t)M * N * 4);
    const int tile_id = m_tile * gridDim.x + n_tile;
    if (threadIdx.x == 0) s_last = atomicAdd(&tickets[tile_id], 1) == splits - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      float* acc_ws = reinterpret_cast<float*>(ws + HEADER_BYTES);
      const int rows = min(BM, M - m0), cols = min(BN, N - n0);
      for (int e = threadIdx.x * 4; e < rows * cols; e += THREADS * 4) {
        const int rr = e / cols, cc = e % cols;
        float4* src = reinterpret_cast<float4*>(acc_ws + (size_t)(m0 + rr) * N + n0 + cc);
        const float4 a = __ldcg(src);
        __half* d = y + (size_t)(m0 + rr) * N + n0 + cc;
        d[0] = __float2half(a.x);
        d[1] = __float2half(a.y);
        d[2] = __float2half(a.z);
        d[3] = __float2half(a.w);
        __stcg(src, make_float4(0.f, 0.f, 0.f, 0.f));
      }
      if (threadIdx.x == 0) tickets[tile_id] = 0;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

struct Plan {
  int tiles_m, tiles_n, splits;
  size_t ws_bytes;
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
  p.ws_bytes = HEADER_BYTES + (sp > 1 ? (size_t)M * N * 4 + (size_t)p.tiles_m * p.tiles_n * 4 : 0);
  return p;
}

}  // namespace mx
}  // namespace b200q

extern "C" {

size_t b200q_mxfp8_workspace_bytes(int64_t M, int64_t N, int64_t K, int device) {
  if (M <= 0 || N <= 0 || K <= 0) return 256;
  return b200q::mx::plan(M, N, K, b200q::num_sms(device)).ws_bytes;
}

int b200q_mxfp8_gemm(const void* a, const void* scales_a, const void* b, const void* scales_b, void* y, int64_t M,
                     int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace b200q;
  using namespace b200q::mx;
  if (M < 0 || N <= 0 || K <= 0) return fail(B200Q_ERR_SHAPE, "mxfp8: M must be >= 0 and N, K > 0");
  if (K % 128) return fail(B200Q_ERR_SHAPE, "mxfp8: K must be a multiple of 128");
  if (N % 32) return fail(B200Q_ERR_ALIGN, "mxfp8: N must be a multiple of 32");
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return fail(B200Q_ERR_SHAPE, "mxfp8: size too large");
  if (M == 0) return B200Q_OK;
  if (!a || !scales_a || !b || !scales_b || !y) return fail(B200Q_ERR_SHAPE, "mxfp8: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(scales_a) | reinterpret_cast<uintptr_t>(scales_b)) & 3)
    return fail(B200Q_ERR_ALIGN, "mxfp8: scale arrays must be 4-byte aligned");
  const Plan p = plan(M, N, K, num_sms(-1));
  if (!workspace || workspace_bytes < p.ws_bytes)
    return fail(B200Q_ERR_WORKSPACE, "mxfp8: workspace of " + std::to_string(p.ws_bytes) + " bytes required");
  CUtensorMap ta, tb;
  int rc;
  if ((rc = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, K, M, (uint64_t)K, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, K, N, (uint64_t)K, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  cudaError_t e = cudaFuncSetAttribute(mxfp8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(mxfp8)");
  dim3 grid(p.tiles_n, p.tiles_m, p.splits);
  mxfp8_tc_kernel<<<grid, THREADS, SMEM, reinterpret_cast<cudaStream_t>(stream)>>>(
      ta, tb, reinterpret_cast<const uint32_t*>(scales_a), reinterpret_cast<const uint32_t*>(scales_b),
      reinterpret_cast<__half*>(y), (int)M, (int)N, (int)K, p.splits, reinterpret_cast<uint8_t*>(workspace));
  return check_cuda(cudaGetLastError(), "mxfp8 launch");
}

}  // extern "C"
