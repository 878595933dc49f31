// Column-sharded W4A16 GEMM whose epilogue is the all-gather, and a
// stand-alone cross-GPU barrier.
//
// Rank r of P computes output columns [col0, col0 + N) of y [M, ldy] and the
// GEMM epilogue stores each finished tile straight into every rank's y over
// NVLink (plain st.global to peer-mapped memory; no multicast), so the
// exchange overlaps the tiles still being computed instead of following the
// GEMM as a separate all-gather and permute.  Given the ranks' signal pads the
// kernel also orders itself against the peers (no rank stores into a peer's
// y before that peer has reached the same call; the call returns only once
// every rank's columns have landed), so one launch is the whole sharded call.
// The pad protocol is described with OutSet in common.cuh; all of its waits
// are bounded and set B200Q_DEV_ERR_TIMEOUT in the workspace status word.
//
// The reference is single-GPU (every task has gpus = 1,
// generate_tasks.py:149); these entry points serve the benchmark's
// column-sharded configuration.
#include <atomic>

#include "common.cuh"

namespace b200q {
int w4a16_decode(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& y,
                 int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream);
int w4a16_tc(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& y,
             int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace, size_t workspace_bytes,
             cudaStream_t stream);

int mxfp8_tc(const void* a, const void* scales_a, const void* b, const void* scales_b, const OutSet& out, int64_t M,
             int64_t N, int64_t K, void* workspace, size_t workspace_bytes, cudaStream_t stream);

namespace {

// The destination set of a column-sharded call: validated peers and pads.
int make_outset(void* const* y_peers, int n_peers, int64_t ldy, int64_t col0, void* const* pads, int rank, int64_t N,
                OutSet* out) {
  if (n_peers < 1 || n_peers > MAX_PEERS) return fail(B200Q_ERR_SHAPE, "peers: need 1..8 destinations");
  if (col0 < 0 || col0 % 32 || ldy % 32 || col0 + N > ldy)
    return fail(B200Q_ERR_ALIGN, "peers: need col0, ldy multiples of 32 and col0 + N <= ldy");
  if (!y_peers) return fail(B200Q_ERR_SHAPE, "peers: null destination array");
  *out = OutSet{};
  for (int i = 0; i < n_peers; ++i) {
    if (!y_peers[i]) return fail(B200Q_ERR_SHAPE, "peers: null destination");
    if (reinterpret_cast<uintptr_t>(y_peers[i]) & 15)
      return fail(B200Q_ERR_ALIGN, "peers: destinations must be 16-byte aligned");
    out->y[i] = y_peers[i];
  }
  if (pads) {
    if (rank < 0 || rank >= n_peers) return fail(B200Q_ERR_SHAPE, "peers: need 0 <= rank < n_peers");
    for (int i = 0; i < n_peers; ++i) {
      if (!pads[i]) return fail(B200Q_ERR_SHAPE, "peers: null signal pad");
      out->pad[i] = reinterpret_cast<uint32_t*>(pads[i]);
    }
    out->world = n_peers;
    out->rank = rank;
  }
  out->n = n_peers;
  out->ldy = (int)ldy;
  out->col0 = (int)col0;
  return B200Q_OK;
}

struct Pads {
  uint32_t* p[MAX_PEERS];
};

// Epoch barrier: bump this rank's barrier counter, publish it to every peer,
// wait for every peer's to reach it.
std::atomic<uint64_t> g_barrier_wait_ns{B200Q_PEER_WAIT_NS};

__global__ void peer_barrier_kernel(Pads pads, int world, int rank, int* status, uint64_t limit_ns) {
  __shared__ uint32_t s_e;
  if (threadIdx.x == 0) {
    const uint32_t e = pads.p[rank][PAD_BARRIER_COUNT] + 1;
    pads.p[rank][PAD_BARRIER_COUNT] = e;
    s_e = e;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int p = threadIdx.x;
  if (p >= world || p == rank) return;
  // everything this stream wrote before (earlier kernels' peer stores
  // included) is ordered before the signal
  asm volatile("fence.sc.sys;" ::: "memory");
  st_release_sys(pads.p[p] + PAD_BARRIER + rank, e);
  if (!wait_epoch(pads.p[rank] + PAD_BARRIER + p, e, limit_ns) && status) atomicOr(status, B200Q_DEV_ERR_TIMEOUT);
}

}  // namespace
}  // namespace b200q

extern "C" {

int64_t b200q_set_peer_barrier_timeout_ms(int64_t ms) {
  const uint64_t ns = ms > 0 ? (uint64_t)ms * 1000000ull : (uint64_t)B200Q_PEER_WAIT_NS;
  return (int64_t)(b200q::g_barrier_wait_ns.exchange(ns) / 1000000ull);
}

int b200q_peer_barrier(void* const* pads, int world, int rank, void* workspace, void* stream) {
  using namespace b200q;
  if (world < 1 || world > MAX_PEERS || rank < 0 || rank >= world)
    return fail(B200Q_ERR_SHAPE, "peer barrier: need 1 <= world <= 8 and 0 <= rank < world");
  if (!pads || !workspace) return fail(B200Q_ERR_SHAPE, "peer barrier: null pointer argument");
  Pads p = {};
  for (int i = 0; i < world; ++i) {
    if (!pads[i]) return fail(B200Q_ERR_SHAPE, "peer barrier: null signal pad");
    p.p[i] = reinterpret_cast<uint32_t*>(pads[i]);
  }
  if (world == 1) return B200Q_OK;
  peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      p, world, rank, reinterpret_cast<int*>(workspace), g_barrier_wait_ns.load());
  return check_cuda(cudaGetLastError(), "peer barrier launch");
}

int b200q_w4a16_gemm_peers(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                           void* const* y_peers, int n_peers, int64_t ldy, int64_t col0, void* const* pads,
                           int rank, int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  using namespace b200q;
  if (dtype != B200Q_DTYPE_FP16 && dtype != B200Q_DTYPE_BF16)
    return fail(B200Q_ERR_UNSUPPORTED, "w4a16: dtype must be fp16 (0) or bf16 (1)");
  if (group != 32 && group != 64 && group != 128 && group != 256)
    return fail(B200Q_ERR_UNSUPPORTED, "w4a16: group must be 32, 64, 128 or 256, got " + std::to_string(group));
  if (M < 0 || N <= 0 || K <= 0) return fail(B200Q_ERR_SHAPE, "w4a16: M must be >= 0 and N, K > 0");
  if (K % group) return fail(B200Q_ERR_SHAPE, "w4a16: K must be a multiple of the group size");
  if (N % 32) return fail(B200Q_ERR_ALIGN, "w4a16: N must be a multiple of 32");
  if (n_peers < 1 || n_peers > MAX_PEERS) return fail(B200Q_ERR_SHAPE, "w4a16 peers: need 1..8 destinations");
  if (col0 < 0 || col0 % 32 || ldy % 32 || col0 + N > ldy)
    return fail(B200Q_ERR_ALIGN, "w4a16 peers: need col0, ldy multiples of 32 and col0 + N <= ldy");
  if (M > (1ll << 30) || ldy > (1ll << 30) || K > (1ll << 30) || M * ldy > (1ll << 40))
    return fail(B200Q_ERR_SHAPE, "w4a16: size too large");
  if (M == 0) return B200Q_OK;
  if (!x || !qweight || !scales || !zeros || !y_peers) return fail(B200Q_ERR_SHAPE, "w4a16: null pointer argument");
  OutSet out = {};
  for (int i = 0; i < n_peers; ++i) {
    if (!y_peers[i]) return fail(B200Q_ERR_SHAPE, "w4a16 peers: null destination");
    if (reinterpret_cast<uintptr_t>(y_peers[i]) & 15)
      return fail(B200Q_ERR_ALIGN, "w4a16 peers: destinations must be 16-byte aligned");
    out.y[i] = y_peers[i];
  }
  if (pads) {
    if (rank < 0 || rank >= n_peers) return fail(B200Q_ERR_SHAPE, "w4a16 peers: need 0 <= rank < n_peers");
    for (int i = 0; i < n_peers; ++i) {
      if (!pads[i]) return fail(B200Q_ERR_SHAPE, "w4a16 peers: null signal pad");
      out.pad[i] = reinterpret_cast<uint32_t*>(pads[i]);
    }
    out.world = n_peers;
    out.rank = rank;
  }
  out.n = n_peers;
  out.ldy = (int)ldy;
  out.col0 = (int)col0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (M >= W4A16_TC_MIN_M)
    return w4a16_tc(x, qweight, scales, zeros, out, M, N, K, group, dtype, workspace, workspace_bytes, st);
  return w4a16_decode(x, qweight, scales, zeros, out, M, N, K, group, dtype, workspace, workspace_bytes, st);
}

int b200q_mxfp8_gemm_peers(const void* a, const void* scales_a, const void* b, const void* scales_b,
                           void* const* y_peers, int n_peers, int64_t ldy, int64_t col0, void* const* pads, int rank,
                           int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace b200q;
  if (M < 0 || N <= 0 || K <= 0) return fail(B200Q_ERR_SHAPE, "mxfp8: M must be >= 0 and N, K > 0");
  if (K % 128) return fail(B200Q_ERR_SHAPE, "mxfp8: K must be a multiple of 128");
  if (N % 32) return fail(B200Q_ERR_ALIGN, "mxfp8: N must be a multiple of 32");
  if (M > (1ll << 30) || ldy > (1ll << 30) || K > (1ll << 30) || M * ldy > (1ll << 40))
    return fail(B200Q_ERR_SHAPE, "mxfp8: size too large");
  if (M == 0) return B200Q_OK;
  if (!a || !scales_a || !b || !scales_b) return fail(B200Q_ERR_SHAPE, "mxfp8: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(scales_a) | reinterpret_cast<uintptr_t>(scales_b)) & 3)
    return fail(B200Q_ERR_ALIGN, "mxfp8: scale arrays must be 4-byte aligned");
  OutSet out;
  int rc = make_outset(y_peers, n_peers, ldy, col0, pads, rank, N, &out);
  if (rc) return rc;
  return mxfp8_tc(a, scales_a, b, scales_b, out, M, N, K, workspace, workspace_bytes,
                  reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
