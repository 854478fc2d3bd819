// Bit packing of ±1 matrices into int32 sign words.
// Contract: quantization/utils/binary_packer.py:4-50 (binary_packer) and
// :53-97 (binary_unpacker): bit j of word w = column 32w+j, bit 1 <=> -1,
// pad columns +1 (bit 0).  Sign convention of functions/binary.py:7-10:
// sign(0) = +1.

#include "common.cuh"

namespace lbx {

// One warp per 32-column word: lane l looks at column 32w+l and the word is
// the warp ballot of "value is -1".
__global__ void pack_kernel(const int8_t *__restrict__ s, int64_t rows, int64_t cols,
                            int64_t wpr, int32_t *__restrict__ out, int32_t *bad) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= rows * wpr) return;
  const int64_t r = gw / wpr, w = gw - r * wpr;
  const int64_t c = w * 32 + lane;
  bool neg = false;
  if (c < cols) {
    const int v = s[r * cols + c];
    neg = v == -1;
    if (bad && v != 1 && v != -1) atomicAdd(bad, 1);
  }
  const uint32_t word = __ballot_sync(0xffffffffu, neg);
  if (lane == 0) out[gw] = (int32_t)word;
}

template <typename T>
__global__ void pack_float_kernel(const T *__restrict__ x, int64_t rows, int64_t cols, int64_t wpr,
                                  int32_t *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= rows * wpr) return;
  const int64_t r = gw / wpr, w = gw - r * wpr;
  const int64_t c = w * 32 + lane;
  bool neg = false;
  if (c < cols) {
    float v;
    if constexpr (sizeof(T) == 4)
      v = x[r * cols + c];
    else
      v = bf16_to_f32(x[r * cols + c]);
    neg = v < 0.f;  // sign(0) = sign(-0) = +1; NaN packs as +1 like the reference cast
  }
  const uint32_t word = __ballot_sync(0xffffffffu, neg);
  if (lane == 0) out[gw] = (int32_t)word;
}

__global__ void unpack_kernel(const int32_t *__restrict__ p, int64_t rows, int64_t cols,
                              int64_t wpr, int8_t *__restrict__ s) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i - r * cols;
  const uint32_t word = (uint32_t)p[r * wpr + (c >> 5)];
  s[i] = (int8_t)(1 - 2 * (int)((word >> (c & 31)) & 1u));
}

}  // namespace lbx

extern "C" int lbx_pack_signs(const int8_t *signs, int64_t rows, int64_t cols, int32_t *packed,
                              int32_t *bad_count, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(rows >= 0 && cols >= 0, "negative shape");
  const int64_t wpr = (cols + 31) / 32;
  const int64_t nw = rows * wpr;
  if (nw == 0) return LBX_OK;
  LBX_CHECK_ARG(signs && packed, "NULL pointer");
  const int warps = 8;
  const int64_t blocks = (nw + warps - 1) / warps;
  pack_kernel<<<(unsigned)blocks, warps * 32, 0, stream>>>(signs, rows, cols, wpr, packed,
                                                            bad_count);
  return cuda_status(cudaGetLastError(), "pack_signs launch");
}

extern "C" int lbx_pack_signs_from_float(const void *w, int32_t w_dtype, int64_t rows,
                                         int64_t cols, int32_t *packed, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(rows >= 0 && cols >= 0, "negative shape");
  LBX_CHECK_ARG(w_dtype == LBX_F32 || w_dtype == LBX_BF16, "bad dtype");
  const int64_t wpr = (cols + 31) / 32;
  const int64_t nw = rows * wpr;
  if (nw == 0) return LBX_OK;
  LBX_CHECK_ARG(w && packed, "NULL pointer");
  const int warps = 8;
  const int64_t blocks = (nw + warps - 1) / warps;
  if (w_dtype == LBX_F32)
    pack_float_kernel<float><<<(unsigned)blocks, warps * 32, 0, stream>>>(
        reinterpret_cast<const float *>(w), rows, cols, wpr, packed);
  else
    pack_float_kernel<uint16_t><<<(unsigned)blocks, warps * 32, 0, stream>>>(
        reinterpret_cast<const uint16_t *>(w), rows, cols, wpr, packed);
  return cuda_status(cudaGetLastError(), "pack_signs_from_float launch");
}

extern "C" int lbx_unpack_signs(const int32_t *packed, int64_t rows, int64_t cols, int8_t *signs,
                                cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(rows >= 0 && cols >= 0, "negative shape");
  const int64_t n = rows * cols;
  if (n == 0) return LBX_OK;
  LBX_CHECK_ARG(signs && packed, "NULL pointer");
  const int64_t wpr = (cols + 31) / 32;
  unpack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(packed, rows, cols, wpr, signs);
  return cuda_status(cudaGetLastError(), "unpack_signs launch");
}
