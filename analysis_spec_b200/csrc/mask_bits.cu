// Bit-packed visibility of a dense additive attention mask, so the drop-in attention
// (transformers hands every layer the same 4-D additive mask, integrations/sdpa_attention.py)
// can run the visibility-bits tensor-core kernel instead of reading the dense mask per layer.
//
// A mask entry is visible iff it is 0 (either sign) and masked iff it is the dtype's lowest
// finite value (torch.finfo(dtype).min, what the reference's masks hold) or -inf; both add
// an exactly-zero probability in the softmax. Any other value makes the mask "not binary"
// (nonbinary[0] = 1) and the bits must not be used. One CTA per mask row, one warp per
// 32-column word (ballot).
#include "common.cuh"

namespace speckv {
namespace {

constexpr int kBitsThreads = 256;

__device__ __forceinline__ void classify(const void* mask, int dtype, long long at, bool& vis, bool& odd) {
  if (dtype == SPECKV_F32) {
    const uint32_t x = static_cast<const uint32_t*>(mask)[at];
    vis = (x & 0x7fffffffu) == 0u;
    odd = !vis && x != 0xff7fffffu && x != 0xff800000u;
  } else {
    const uint16_t x = static_cast<const uint16_t*>(mask)[at];
    const uint16_t lowest = dtype == SPECKV_BF16 ? 0xff7fu : 0xfbffu;
    const uint16_t ninf = dtype == SPECKV_BF16 ? 0xff80u : 0xfc00u;
    vis = (x & 0x7fffu) == 0u;
    odd = !vis && x != lowest && x != ninf;
  }
}

__global__ void __launch_bounds__(kBitsThreads) mask_bits_kernel(const void* __restrict__ mask, int dtype,
                                                                 long long rows, long long cols, long long sb,
                                                                 long long sr, long long sc,
                                                                 uint32_t* __restrict__ bits, long long row_words,
                                                                 int* __restrict__ first_col,
                                                                 int* __restrict__ nonbinary) {
  const long long row = blockIdx.x;  // b * rows + r
  const long long b = row / rows, r = row % rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int first = 0x7fffffff;
  bool any_odd = false;
  for (long long w = warp; w < row_words; w += kBitsThreads / 32) {
    const long long c = w * 32 + lane;
    bool vis = false, odd = false;
    if (c < cols) classify(mask, dtype, b * sb + r * sr + c * sc, vis, odd);
    any_odd |= odd;
    const uint32_t word = __ballot_sync(0xffffffffu, vis);
    if (lane == 0) {
      bits[row * row_words + w] = word;
      if (word != 0u && first == 0x7fffffff) first = (int)(w * 32 + __ffs(word) - 1);
    }
  }
  if (lane == 0 && first != 0x7fffffff) atomicMin(first_col + b, first);
  if (__any_sync(0xffffffffu, any_odd) && lane == 0) *nonbinary = 1;
}

}  // namespace
}  // namespace speckv

using namespace speckv;

extern "C" int speckv_mask_bits(const void* mask, int32_t dtype, int64_t batch, int64_t rows, int64_t columns,
                                const int64_t* mask_strides, uint32_t* bits, int64_t row_words, int32_t* first_col,
                                int32_t* nonbinary, void* stream) {
  const char* fn = "speckv_mask_bits";
  if (batch < 0 || rows < 0 || columns < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (dtype != SPECKV_F32 && dtype != SPECKV_BF16 && dtype != SPECKV_F16)
    return fail(SPECKV_EINVAL, "%s: unsupported mask dtype %d", fn, dtype);
  if (row_words < (columns + 31) / 32)
    return fail(SPECKV_EINVAL, "%s: %lld words per row < %lld columns", fn, (long long)row_words,
                (long long)columns);
  if (batch * rows == 0) return SPECKV_OK;
  if (!mask || !mask_strides || !bits || !first_col || !nonbinary) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (batch * rows > 0x7fffffffll) return fail(SPECKV_ENOSUPPORT, "%s: too many mask rows", fn);
  const int dst = check_current_device(fn, {mask, bits, first_col, nonbinary});
  if (dst) return dst;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // first_col starts above any column (atomicMin), the flag at 0
  if (cudaMemsetAsync(first_col, 0x7f, (size_t)batch * sizeof(int32_t), s) != cudaSuccess ||
      cudaMemsetAsync(nonbinary, 0, sizeof(int32_t), s) != cudaSuccess)
    return fail(SPECKV_ECUDA, "%s: cudaMemsetAsync failed", fn);
  mask_bits_kernel<<<(unsigned)(batch * rows), kBitsThreads, 0, s>>>(mask, dtype, rows, columns, mask_strides[0],
                                                                     mask_strides[1], mask_strides[2], bits,
                                                                     row_words, first_col, nonbinary);
  return check_launch(fn);
}
