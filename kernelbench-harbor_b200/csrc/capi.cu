// extern "C" entry points: argument validation and dispatch to the kernels.
#include "common.cuh"

namespace b200q {
size_t w4a16_decode_ws_bytes(int64_t M, int64_t N, int64_t K, int device);
int w4a16_decode(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& y,
                 int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream);
size_t w4a16_tc_ws_bytes(int64_t M, int64_t N, int64_t K, int device);
int w4a16_tc(const void* x, const int32_t* qweight, const void* scales, const void* zeros, const OutSet& y,
             int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace, size_t workspace_bytes,
             cudaStream_t stream);

int w4a16_tc_grouped(const void* x, const int32_t* qw, const void* sc, const void* zr, const int32_t* qw2,
                     const void* sc2, const void* zr2, const int32_t* offsets, int64_t E, void* y, int64_t rows,
                     int64_t N, int64_t K, int64_t group, int dtype, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream);

size_t w8a8_ws_bytes(int64_t M, int64_t N, int64_t K, int device);
int w8a8_tc(const void* x_int8, const void* w_int8, const void* x_scale, const void* w_scale, void* y, int64_t M,
            int64_t N, int64_t K, void* workspace, size_t workspace_bytes, cudaStream_t stream);


static int check_w4a16_shape(int64_t M, int64_t N, int64_t K, int64_t group, int dtype) {
  if (dtype != B200Q_DTYPE_FP16 && dtype != B200Q_DTYPE_BF16)
    return fail(B200Q_ERR_UNSUPPORTED, "w4a16: dtype must be fp16 (0) or bf16 (1)");
  if (group != 32 && group != 64 && group != 128 && group != 256)
    return fail(B200Q_ERR_UNSUPPORTED, "w4a16: group must be 32, 64, 128 or 256, got " + std::to_string(group));
  if (M < 0 || N <= 0 || K <= 0) return fail(B200Q_ERR_SHAPE, "w4a16: M must be >= 0 and N, K > 0");
  if (K % group) return fail(B200Q_ERR_SHAPE, "w4a16: K must be a multiple of the group size");
  if (N % 32)
    return fail(B200Q_ERR_ALIGN, "w4a16: N must be a multiple of 32 (qweight rows must be 16-byte pitched)");
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return fail(B200Q_ERR_SHAPE, "w4a16: size too large");
  return B200Q_OK;
}
}  // namespace b200q

extern "C" {

size_t b200q_w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group, int device) {
  (void)group;
  if (M <= 0 || N <= 0 || K <= 0) return 256;
  if (M >= b200q::W4A16_TC_MIN_M)
    return b200q::w4a16_tc_ws_bytes(M, N, K, device);
  return b200q::w4a16_decode_ws_bytes(M, N, K, device);
}

int b200q_w4a16_gemm(const void* x, const int32_t* qweight, const void* scales, const void* zeros, void* y,
                     int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                     size_t workspace_bytes, void* stream) {
  using namespace b200q;
  int rc = check_w4a16_shape(M, N, K, group, dtype);
  if (rc) return rc;
  if (M == 0) return B200Q_OK;
  if (!x || !qweight || !scales || !zeros || !y) return fail(B200Q_ERR_SHAPE, "w4a16: null pointer argument");
  if (reinterpret_cast<uintptr_t>(y) & 15) return fail(B200Q_ERR_ALIGN, "w4a16: y must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (M >= W4A16_TC_MIN_M)
    return w4a16_tc(x, qweight, scales, zeros, single_out(y, N), M, N, K, group, dtype, workspace, workspace_bytes, st);
  return w4a16_decode(x, qweight, scales, zeros, single_out(y, N), M, N, K, group, dtype, workspace, workspace_bytes, st);
}

int b200q_moe_grouped_gemm(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                           const int32_t* qweight_up, const void* scales_up, const void* zeros_up,
                           const int32_t* offsets, int64_t E, void* y, int64_t rows, int64_t N, int64_t K,
                           int64_t group, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace b200q;
  int rc = check_w4a16_shape(rows, N, K, group, dtype);
  if (rc) return rc;
  if (E < 1 || E > 64) return fail(B200Q_ERR_SHAPE, "moe_grouped_gemm: need 1 <= E <= 64");
  if (K % 64) return fail(B200Q_ERR_ALIGN, "moe_grouped_gemm: K must be a multiple of 64");
  if (E * K > (1ll << 31) - 1) return fail(B200Q_ERR_SHAPE, "moe_grouped_gemm: E*K too large");
  const bool glu = qweight_up || scales_up || zeros_up;
  if (glu && !(qweight_up && scales_up && zeros_up))
    return fail(B200Q_ERR_SHAPE, "moe_grouped_gemm: give all three up-projection arrays or none");
  if (rows == 0) return B200Q_OK;
  if (!x || !qweight || !scales || !zeros || !offsets || !y)
    return fail(B200Q_ERR_SHAPE, "moe_grouped_gemm: null pointer argument");
  return w4a16_tc_grouped(x, qweight, scales, zeros, qweight_up, scales_up, zeros_up, offsets, E, y, rows, N, K,
                          group, dtype, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t b200q_w8a8_workspace_bytes(int64_t M, int64_t N, int64_t K, int device) {
  if (M <= 0 || N <= 0 || K <= 0) return 256;
  return b200q::w8a8_ws_bytes(M, N, K, device);
}

int b200q_w8a8_gemm(const void* x_int8, const void* w_int8, const void* x_scale, const void* w_scale, void* y,
                    int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace b200q;
  if (M < 0 || N <= 0 || K <= 0) return fail(B200Q_ERR_SHAPE, "w8a8: M must be >= 0 and N, K > 0");
  if (K % 16) return fail(B200Q_ERR_ALIGN, "w8a8: K must be a multiple of 16 (x rows must be 16-byte pitched)");
  if (N % 32) return fail(B200Q_ERR_ALIGN, "w8a8: N must be a multiple of 32");
  if (M > (1ll << 30) || N > (1ll << 30) || K > 130000) return fail(B200Q_ERR_SHAPE, "w8a8: size too large");
  if (M == 0) return B200Q_OK;
  if (!x_int8 || !w_int8 || !x_scale || !w_scale || !y) return fail(B200Q_ERR_SHAPE, "w8a8: null pointer argument");
  return w8a8_tc(x_int8, w_int8, x_scale, w_scale, y, M, N, K, workspace, workspace_bytes,
                 reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
