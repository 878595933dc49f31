// b200q_w4a16_gemm_noalloc: the small-M (decode) W4A16 GEMM for callers that
// cannot allocate device memory.
//
// Some callers have no allocator to hand: a plugin loaded into a host program
// that owns every cudaMalloc (and may forbid new ones after start-up), code
// running under a fixed memory budget, or a C caller that wants one call with
// no workspace bookkeeping.  For them this entry point takes only inputs and
// outputs; the decode kernel's split-K scratch lives in the file-scope device
// array below instead of a caller workspace.
//
// Properties a user must know:
//  * The array is NOALLOC_SCRATCH_BYTES (8 MiB) of device memory on every GPU
//    that loads this library, held until the process exits.
//  * Shapes whose scratch would exceed it, and M outside [1, 32], are rejected
//    with B200Q_ERR_SHAPE and a message; nothing is launched then.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * Every call shares the one array: calls that can overlap on the GPU (two
//    streams, or two host threads) race and give wrong results.  Serialise them.
//  * Nothing is allocated or freed: no cudaMalloc/cudaFree and no allocating
//    library routine.  Each call clears the array's header and split-K tickets
//    (cudaMemsetAsync on the caller's stream) before the kernel runs.
//  * A device-side error (a bounded wait that gave up) is recorded in the
//    array's header word; b200q_w4a16_noalloc_status reads and clears it.  The
//    next call clears it too, so read it before the next call.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace b200q {
size_t w4a16_decode_ws_bytes(int64_t M, int64_t N, int64_t K, int device);
int w4a16_decode(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& y,
                 int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream);
}  // namespace b200q

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 8u << 20;

static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch per device.  In host code the symbol is
// only a stand-in; the kernel must receive the address looked up here.
int scratch_address(int device, void** out) {
  static std::mutex mu;
  static std::vector<void*> addr;
  std::lock_guard<std::mutex> lk(mu);
  if (device >= (int)addr.size()) addr.resize(device + 1, nullptr);
  if (!addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return b200q::fail(B200Q_ERR_CUDA, std::string("cudaGetSymbolAddress(noalloc scratch): ") +
                                            cudaGetErrorString(e));
    addr[device] = p;
  }
  *out = addr[device];
  return B200Q_OK;
}

}  // namespace

extern "C" int b200q_w4a16_gemm_noalloc(const void* x, const int32_t* qweight, const void* scales,
                                        const void* zeros, void* y, int64_t M, int64_t N, int64_t K,
                                        int64_t group, int dtype, void* stream) {
  using namespace b200q;
  if (M < 1 || M > 32)
    return fail(B200Q_ERR_SHAPE, "w4a16 noalloc: M must be in [1, 32] (the decode path), got " + std::to_string(M));
  if (dtype != B200Q_DTYPE_FP16 && dtype != B200Q_DTYPE_BF16)
    return fail(B200Q_ERR_UNSUPPORTED, "w4a16 noalloc: dtype must be fp16 (0) or bf16 (1)");
  if (group != 32 && group != 64 && group != 128 && group != 256)
    return fail(B200Q_ERR_UNSUPPORTED, "w4a16 noalloc: group must be 32, 64, 128 or 256");
  if (N <= 0 || K <= 0 || K % group) return fail(B200Q_ERR_SHAPE, "w4a16 noalloc: N, K > 0 and K % group == 0");
  if (N % 32) return fail(B200Q_ERR_ALIGN, "w4a16 noalloc: N must be a multiple of 32");
  if (N > (1ll << 30) || K > (1ll << 30)) return fail(B200Q_ERR_SHAPE, "w4a16 noalloc: size too large");
  if (!x || !qweight || !scales || !zeros || !y) return fail(B200Q_ERR_SHAPE, "w4a16 noalloc: null pointer");
  if (reinterpret_cast<uintptr_t>(y) & 15) return fail(B200Q_ERR_ALIGN, "w4a16 noalloc: y must be 16-byte aligned");
  int device = 0;
  int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice");
  if (rc) return rc;
  const size_t need = w4a16_decode_ws_bytes(M, N, K, device);
  if (need > NOALLOC_SCRATCH_BYTES)
    return fail(B200Q_ERR_SHAPE, "w4a16 noalloc: this shape needs " + std::to_string(need) +
                                     " bytes of scratch, more than the fixed " +
                                     std::to_string(NOALLOC_SCRATCH_BYTES) + " bytes");
  void* scratch = nullptr;
  if ((rc = scratch_address(device, &scratch))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // cleared before each call: the 256-byte status header and the split-K
  // counters (two per 256-column strip and 16-row chunk, at most 2 chunks); the kernel
  // overwrites its partial slots before reading them and zeroes them after
  const size_t tickets = ((size_t)2 * ((N + 255) / 256) * 8 + 255) & ~size_t(255);
  const size_t clear = need < 256 + tickets ? need : 256 + tickets;
  if ((rc = check_cuda(cudaMemsetAsync(scratch, 0, clear, st), "noalloc scratch clear"))) return rc;
  return w4a16_decode(x, qweight, scales, zeros, single_out(y, N), M, N, K, group, dtype, scratch, NOALLOC_SCRATCH_BYTES, st);
}

extern "C" int b200q_w4a16_noalloc_status(void* stream) {
  using namespace b200q;
  int device = 0;
  int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice");
  if (rc) return rc;
  void* scratch = nullptr;
  if ((rc = scratch_address(device, &scratch))) return rc;
  return b200q_workspace_status(scratch, stream);
}
