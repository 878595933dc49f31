// W8A8 GEMM on the tcgen05 tensor cores (kind::i8): the sibling of the W4A16
// path for W8A8_REF (generate_tasks.py:198-215):
//   y[M, N] = fp16( (x_int8[M, K] . w_int8[K, N])  * x_scale[M] * w_scale[N] )
// with exact int32 accumulation (|acc| <= K * 127^2 < 2^31 for K < 133,000) in
// tensor memory and the rescale in fp32 in the order the reference applies it
// ((acc * x_scale) * w_scale).  The reference accumulates in fp32, whose
// rounding this kernel does not reproduce: it is exact instead.
//
// Layouts are the reference's: x_int8 [M, K] (K-major A operand), w_int8
// [K, N] (N contiguous: the MN-major B operand, read by TMA as is, no
// re-layout), x_scale [M] and w_scale [N] fp16.
//
// One CTA: a 128 x 256 output tile over a K range (split-K when the tiles
// cannot fill the SMs; partial sums are exact int32, added with atomics, so
// the result does not depend on their order).  Warp 0: TMA producer (x box
// [128 x 128 k], two w boxes [128 k x 128 n], 4-deep ring); warp 1: TMEM owner
// and MMA issuer (4 x M128 N256 K32 per 128-deep stage); warps 2..5: epilogue.
#include "common.cuh"

namespace b200q {
namespace w8 {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int THREADS = 6 * 32;
constexpr uint32_t X_BYTES = BM * BK;      // 16 KB
constexpr uint32_t WH_BYTES = BK * 128;    // one 128-column half of the w tile: 16 KB
constexpr uint32_t STAGE = X_BYTES + 2 * WH_BYTES;
constexpr uint32_t OFF_BAR = STAGES * STAGE;
constexpr uint32_t SMEM = OFF_BAR + 256 + 1024;
constexpr int HEADER_BYTES = 256;
constexpr int MAX_SPLITS = 16;
static_assert(SMEM <= 227 * 1024, "shared memory budget");

__global__ void __launch_bounds__(THREADS, 1)
    w8a8_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __half* __restrict__ x_scale, const __half* __restrict__ w_scale, __half* __restrict__ y,
                   int M, int N, int K, int splits, uint8_t* __restrict__ ws) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ int s_err, s_last;

  int* status = reinterpret_cast<int*>(ws);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z;
  const int n0 = n_tile * BN, m0 = m_tile * BM;
  const int nk_total = (K + BK - 1) / BK;
  const int k_begin = (int)((long long)split * nk_total / splits);
  const int nk = (int)((long long)(split + 1) * nk_total / splits) - k_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
    s_err = 0;
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
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
        tma_load_2d(st, &tm_x, kb, m0, &full[s]);
        tma_load_2d(st + X_BYTES, &tm_w, n0, kb, &full[s]);
        tma_load_2d(st + X_BYTES + WH_BYTES, &tm_w, n0 + 128, kb, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(BM, BN, /*a_mn=*/0, /*b_mn=*/1);
      for (int it = 0; it < nk; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, status)) {
          s_err = 1;
          break;
        }
        tc_fence_after();
        const uint32_t xa = smem_u32(smem + s * STAGE);
        const uint32_t wa = xa + X_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk) {
          // A: K-major (32 int8 = 32 B per MMA step), 8-row groups 1024 B apart.
          // B: MN-major, 128-column atoms 16 KB apart (the two TMA boxes),
          //    8-row K groups 1024 B apart; 32 K rows per MMA step = 4096 B.
          const uint64_t ad = smem_desc(xa + kk * 32, 16, 1024, 2);
          const uint64_t bd = smem_desc(wa + kk * 4096, WH_BYTES, 1024, 2);
          tc_mma_i8_ss(tmem, ad, bd, idesc, (it | kk) != 0);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    if (mbar_wait(acc_full, 0, status)) {
      tc_fence_after();
      const int qd = warp & 3;
      const int row = m0 + qd * 32 + lane;
      const float xs = row < M ? __half2float(x_scale[row]) : 0.f;
      int* acc_ws = reinterpret_cast<int*>(ws + HEADER_BYTES);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(qd * 32) << 16) + c0, r);
        tmem_ld_wait();
        const int col = n0 + c0;
        if (row >= M || col >= N) continue;
        if (splits == 1) {
          uint32_t packed[16];
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            const float a = (float)(int)r[2 * p] * xs * __half2float(w_scale[col + 2 * p]);
            const float b = (float)(int)r[2 * p + 1] * xs * __half2float(w_scale[col + 2 * p + 1]);
            __half2 h = __floats2half2_rn(a, b);
            packed[p] = *reinterpret_cast<uint32_t*>(&h);
          }
          uint4* dst = reinterpret_cast<uint4*>(y + (size_t)row * N + col);
#pragma unroll
          for (int p = 0; p < 4; ++p)
            dst[p] = make_uint4(packed[4 * p], packed[4 * p + 1], packed[4 * p + 2], packed[4 * p + 3]);
        } else {
          int* dst = acc_ws + (size_t)row * N + col;
#pragma unroll
          for (int p = 0; p < 32; ++p) atomicAdd(dst + p, (int)r[p]);
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
      int* acc_ws = reinterpret_cast<int*>(ws + HEADER_BYTES);
      const int rows = min(BM, M - m0), cols = min(BN, N - n0);
      for (int e = threadIdx.x * 4; e < rows * cols; e += THREADS * 4) {
        const int rr = e / cols, cc = e % cols;  // cols % 16 == 0: an int4 never straddles rows
        int4* src = reinterpret_cast<int4*>(acc_ws + (size_t)(m0 + rr) * N + n0 + cc);
        const int4 a = __ldcg(src);
        const float xs = __half2float(x_scale[m0 + rr]);
        __half* d = y + (size_t)(m0 + rr) * N + n0 + cc;
        d[0] = __float2half((float)a.x * xs * __half2float(w_scale[n0 + cc]));
        d[1] = __float2half((float)a.y * xs * __half2float(w_scale[n0 + cc + 1]));
        d[2] = __float2half((float)a.z * xs * __half2float(w_scale[n0 + cc + 2]));
        d[3] = __float2half((float)a.w * xs * __half2float(w_scale[n0 + cc + 3]));
        __stcg(src, make_int4(0, 0, 0, 0));
      }
      if (threadIdx.x == 0) tickets[tile_id] = 0;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
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
  const int nk = (int)((K + BK - 1) / BK);
  int sp = sms / (p.tiles_m * p.tiles_n);
  if (sp < 1) sp = 1;
  if (sp > MAX_SPLITS) sp = MAX_SPLITS;
  if (sp > nk / 2) sp = nk / 2 > 0 ? nk / 2 : 1;
  p.splits = sp;
  p.ws_bytes = HEADER_BYTES + (sp > 1 ? (size_t)M * N * 4 + (size_t)p.tiles_m * p.tiles_n * 4 : 0);
  return p;
}

}  // namespace w8

size_t w8a8_ws_bytes(int64_t M, int64_t N, int64_t K, int device) {
  return w8::plan(M, N, K, num_sms(device)).ws_bytes;
}

int w8a8_tc(const void* x_int8, const void* w_int8, const void* x_scale, const void* w_scale, void* y, int64_t M,
            int64_t N, int64_t K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace w8;
  const Plan p = plan(M, N, K, num_sms(-1));
  if (!workspace || workspace_bytes < p.ws_bytes)
    return fail(B200Q_ERR_WORKSPACE, "w8a8: workspace of " + std::to_string(p.ws_bytes) + " bytes required");
  CUtensorMap tx, tw;
  int rc;
  if ((rc = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_int8, K, M, (uint64_t)K, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_int8, N, K, (uint64_t)N, 128, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  cudaError_t e = cudaFuncSetAttribute(w8a8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(w8a8)");
  dim3 grid(p.tiles_n, p.tiles_m, p.splits);
  w8a8_tc_kernel<<<grid, THREADS, SMEM, stream>>>(tx, tw, reinterpret_cast<const __half*>(x_scale),
                                                   reinterpret_cast<const __half*>(w_scale),
                                                   reinterpret_cast<__half*>(y), (int)M, (int)N, (int)K, p.splits,
                                                   reinterpret_cast<uint8_t*>(workspace));
  return check_cuda(cudaGetLastError(), "w8a8 launch");
}

}  // namespace b200q
