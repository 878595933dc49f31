// GPU weight packer: 4-bit codes -> the reference's packed qweight layout.
//
// qweight[k, j] = sum_i ((codes[k, 8j + i] + offset) & 0xF) << 4i  (int32),
// the packing loop of QUANT_REF.get_inputs (generate_tasks.py:65-69): nibble i
// of word j holds column 8j + i.  offset = 0 packs unsigned codes in [0, 15]
// (the reference's own format); offset = 8 packs the signed symmetric int4
// weights of FUSED_QMOE_REF / LORA_REF (int8 in [-8, 7], generate_tasks.py:385,
// 414) as unsigned codes with zero point 8, so that the asymmetric W4A16
// kernels compute (q + 8 - 8) * s = q * s exactly as those modules dequantise.
// Codes outside the 4-bit range set B200Q_DEV_ERR_BOUNDS in the status word
// (when one is given) and are masked.
#include "common.cuh"

namespace b200q {
namespace {

__global__ void pack_int4_kernel(const int8_t* __restrict__ codes, int64_t words_per_row, int64_t total_words,
                                 int offset, int32_t* __restrict__ out, int* status) {
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total_words;
       w += (int64_t)gridDim.x * blockDim.x) {
    const uint2 v = reinterpret_cast<const uint2*>(codes)[w];  // 8 consecutive codes of one row
    uint32_t word = 0;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t src = i < 4 ? v.x : v.y;
      const int c = (int)(int8_t)((src >> (8 * (i & 3))) & 0xFF) + offset;
      bad |= (c < 0) | (c > 15);
      word |= (uint32_t)(c & 0xF) << (4 * i);
    }
    out[w] = (int32_t)word;
    if (bad && status) atomicOr(status, B200Q_DEV_ERR_BOUNDS);
  }
  (void)words_per_row;
}

}  // namespace
}  // namespace b200q

extern "C" int b200q_pack_int4(const void* codes, int64_t K, int64_t N, int offset, int32_t* qweight,
                               void* workspace, void* stream) {
  using namespace b200q;
  if (K < 0 || N <= 0 || N % 8) return fail(B200Q_ERR_SHAPE, "pack_int4: N must be a positive multiple of 8");
  if (offset != 0 && offset != 8) return fail(B200Q_ERR_UNSUPPORTED, "pack_int4: offset must be 0 or 8");
  if (K == 0) return B200Q_OK;
  if (!codes || !qweight) return fail(B200Q_ERR_SHAPE, "pack_int4: null pointer argument");
  if (reinterpret_cast<uintptr_t>(codes) & 7)
    return fail(B200Q_ERR_ALIGN, "pack_int4: codes must be 8-byte aligned");
  const int64_t words = K * (N / 8);
  const int threads = 256;
  int64_t blocks = (words + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms(-1) * 16;
  if (blocks > cap) blocks = cap;
  pack_int4_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const int8_t*>(codes), N / 8, words, offset, qweight, reinterpret_cast<int*>(workspace));
  return check_cuda(cudaGetLastError(), "pack_int4 launch");
}
