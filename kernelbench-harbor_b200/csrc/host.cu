// Host-side plumbing shared by every entry point: error strings, device
// properties, tensor-map encoding through the driver entry point, the device
// status word.
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace b200q {

static thread_local std::string g_last_error;
static std::atomic<int> g_weight_prefetch{0};

bool weight_prefetch_enabled() { return g_weight_prefetch.load(std::memory_order_relaxed) != 0; }

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B200Q_OK;
  return fail(B200Q_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int num_sms(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lk(mu);
  if (device < 0) device = current_device();
  if (device >= (int)cache.size()) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(B200Q_ERR_ALIGN, "tensor base address is not 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    return fail(B200Q_ERR_ALIGN, "row pitch " + std::to_string(row_stride_bytes) +
                                     " bytes is not a multiple of 16 (TMA rule)");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
  return B200Q_OK;
}

int encode_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
              CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(B200Q_ERR_ALIGN, "tensor base address is not 16-byte aligned");
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    return fail(B200Q_ERR_ALIGN, "tensor strides are not multiples of 16 bytes (TMA rule)");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled (3d) failed with CUresult " + std::to_string((int)r));
  return B200Q_OK;
}

}  // namespace b200q

extern "C" {

int b200q_version(void) { return (0 << 16) | 2; }

int b200q_set_weight_prefetch(int enable) {
  const int old = b200q::g_weight_prefetch.exchange(enable ? 1 : 0);
  return old;
}

const char* b200q_last_error(void) { return b200q::g_last_error.c_str(); }

int b200q_workspace_status(void* workspace, void* stream) {
  if (!workspace) return b200q::fail(B200Q_ERR_WORKSPACE, "workspace is null");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int host = 0;
  int rc = b200q::check_cuda(cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, s),
                             "status copy");
  if (rc) return rc;
  rc = b200q::check_cuda(cudaStreamSynchronize(s), "status sync");
  if (rc) return rc;
  if (host != 0) {
    rc = b200q::check_cuda(cudaMemsetAsync(workspace, 0, sizeof(int), s), "status clear");
    if (rc) return rc;
    cudaStreamSynchronize(s);
  }
  return host;
}

}  // extern "C"
