// Additive masks of the draft model's attention: the causal mask of the draft commit
// (AttentionWorkspace.causal, helper/opd_attention.py:31-43 with the kernel of
// helper/opd_attention_kernels.py:7-22) and the mask of each draft expansion step
// (helper/opd_generate.py:143-162). Visible entries are 0, the others the dtype's
// lowest finite value (torch.finfo(dtype).min): -FLT_MAX (0xff7fffff), bf16 0xff7f,
// fp16 -65504 (0xfbff). One CTA per (mask row, 1024-column chunk).
#include "common.cuh"

namespace speckv {
namespace {

constexpr int kDraftThreads = 256;
constexpr int kDraftCols = 1024;

__device__ __forceinline__ void put(void* mask, int dtype, long long at, bool vis) {
  if (dtype == SPECKV_F32) {
    static_cast<uint32_t*>(mask)[at] = vis ? 0u : 0xff7fffffu;
  } else if (dtype == SPECKV_BF16) {
    static_cast<uint16_t*>(mask)[at] = vis ? (uint16_t)0 : (uint16_t)0xff7f;
  } else {
    static_cast<uint16_t*>(mask)[at] = vis ? (uint16_t)0 : (uint16_t)0xfbff;
  }
}

// Optional visibility bits of the same mask (the form the tensor-core attention reads):
// bits[row][w] bit i = entry (row, 32 w + i) is visible, words up to row_words (zero past
// the last column), and first_col[b] lowered (atomicMin) to the first visible column of
// any row of sequence b. Each warp covers 32 consecutive columns per iteration (ballot).
__device__ __forceinline__ void emit_bits(bool vis, long long c, long long row, long long b, uint32_t* bits,
                                          long long row_words, int* first_col, int& first) {
  const uint32_t word = __ballot_sync(0xffffffffu, vis);
  if ((threadIdx.x & 31) == 0 && bits != nullptr) {
    const long long w = c >> 5;
    if (w < row_words) bits[row * row_words + w] = word;
    if (word != 0u && first == 0x7fffffff) first = (int)(c + __ffs(word) - 1);
  }
}

__device__ __forceinline__ void flush_first(int first, long long b, int* first_col) {
  if ((threadIdx.x & 31) == 0 && first_col != nullptr && first != 0x7fffffff) atomicMin(first_col + b, first);
}

// mask (batch, 1, query, columns): row r of sequence b sees columns c <= past + r that
// are not padding.
__global__ void __launch_bounds__(kDraftThreads) causal_mask_kernel(void* mask, int dtype, long long query,
                                                                    long long past, long long columns,
                                                                    const uint8_t* __restrict__ pad, long long ps0,
                                                                    long long ps1, uint32_t* bits, long long row_words,
                                                                    int* first_col) {
  const long long row = blockIdx.x;  // b * query + r
  const long long b = row / query, r = row % query;
  const long long c0 = (long long)blockIdx.y * kDraftCols;
  int first = 0x7fffffff;
  for (int k = 0; k < kDraftCols / kDraftThreads; ++k) {
    const long long c = c0 + k * kDraftThreads + threadIdx.x;
    bool vis = false;
    if (c < columns) {
      vis = c <= past + r;
      if (pad != nullptr && pad[b * ps0 + c * ps1]) vis = false;
      put(mask, dtype, row * columns + c, vis);
    }
    emit_bits(vis, c - (threadIdx.x & 31), row, b, bits, row_words, first_col, first);
  }
  flush_first(first, b, first_col);
}

// mask (batch, 1, query, columns): row r of sequence b sees the columns below `init`
// and its own column seen[b][r] (zero, then [init:] = min, then the scatter of 0),
// padding columns off last.
__global__ void __launch_bounds__(kDraftThreads) expansion_mask_kernel(void* mask, int dtype, long long query,
                                                                       long long columns, long long init,
                                                                       const int64_t* __restrict__ seen,
                                                                       long long ss0, long long ss1,
                                                                       const uint8_t* __restrict__ pad,
                                                                       long long ps0, long long ps1,
                                                                       unsigned long long* err, uint32_t* bits,
                                                                       long long row_words, int* first_col) {
  const long long row = blockIdx.x;
  const long long b = row / query, r = row % query;
  const long long own = seen[b * ss0 + r * ss1];
  if (own < 0 || own >= columns) {  // the reference's scatter_ would raise: report, keep the rest
    if (threadIdx.x == 0 && blockIdx.y == 0) record_error(err, SPECKV_DERR_SEEN_INDEX, own);
  }
  const long long c0 = (long long)blockIdx.y * kDraftCols;
  int first = 0x7fffffff;
  for (int k = 0; k < kDraftCols / kDraftThreads; ++k) {
    const long long c = c0 + k * kDraftThreads + threadIdx.x;
    bool vis = false;
    if (c < columns) {
      vis = c < init || c == own;
      if (pad != nullptr && pad[b * ps0 + c * ps1]) vis = false;
      put(mask, dtype, row * columns + c, vis);
    }
    emit_bits(vis, c - (threadIdx.x & 31), row, b, bits, row_words, first_col, first);
  }
  flush_first(first, b, first_col);
}

int check_mask(const char* fn, void* mask, int32_t dtype, int64_t batch, int64_t query, int64_t columns) {
  if (batch < 0 || query < 0 || columns < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (dtype != SPECKV_F32 && dtype != SPECKV_BF16 && dtype != SPECKV_F16)
    return fail(SPECKV_EINVAL, "%s: unsupported mask dtype %d", fn, dtype);
  if (batch * query != 0 && columns != 0 && mask == nullptr) return fail(SPECKV_EINVAL, "%s: null mask", fn);
  if (batch * query > 0x7fffffffll) return fail(SPECKV_ENOSUPPORT, "%s: too many mask rows", fn);
  if ((columns + kDraftCols - 1) / kDraftCols > 65535) return fail(SPECKV_ENOSUPPORT, "%s: too many columns", fn);
  return SPECKV_OK;
}

// bits and first_col come together; first_col starts above any column (atomicMin).
int check_bits(const char* fn, int64_t batch, int64_t columns, uint32_t* bits, int64_t row_words, int32_t* first_col,
               cudaStream_t s) {
  if (bits == nullptr) return SPECKV_OK;
  if (first_col == nullptr) return fail(SPECKV_EINVAL, "%s: visibility bits without first_col", fn);
  if (row_words < 4 * ((columns + 127) / 128))
    return fail(SPECKV_EINVAL, "%s: row_words %lld below 4 * ceil(columns / 128)", fn, (long long)row_words);
  if (cudaMemsetAsync(first_col, 0x7f, (size_t)batch * sizeof(int32_t), s) != cudaSuccess)
    return fail(SPECKV_ECUDA, "%s: cudaMemsetAsync failed", fn);
  return SPECKV_OK;
}

}  // namespace
}  // namespace speckv

using namespace speckv;

extern "C" int speckv_causal_mask(void* mask, int32_t dtype, int64_t batch, int64_t query, int64_t past,
                                  int64_t columns, const uint8_t* pad, int64_t pad_stride_b, int64_t pad_stride_c,
                                  uint32_t* bits, int64_t row_words, int32_t* first_col, void* stream) {
  const char* fn = "speckv_causal_mask";
  int st = check_mask(fn, mask, dtype, batch, query, columns);
  if (st) return st;
  if (past < 0) return fail(SPECKV_EINVAL, "%s: negative past", fn);
  if (batch * query == 0 || columns == 0) return SPECKV_OK;
  st = check_current_device(fn, {mask, pad, bits, first_col});
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = check_bits(fn, batch, columns, bits, row_words, first_col, s);
  if (st) return st;
  dim3 grid((unsigned)(batch * query), (unsigned)((columns + kDraftCols - 1) / kDraftCols));
  causal_mask_kernel<<<grid, kDraftThreads, 0, s>>>(mask, dtype, query, past, columns, pad, pad_stride_b,
                                                    pad_stride_c, bits, row_words, first_col);
  return check_launch(fn);
}

extern "C" int speckv_expansion_mask(void* mask, int32_t dtype, int64_t batch, int64_t query, int64_t columns,
                                     int64_t init_length, const int64_t* seen, int64_t seen_stride_b,
                                     int64_t seen_stride_r, const uint8_t* pad, int64_t pad_stride_b,
                                     int64_t pad_stride_c, uint32_t* bits, int64_t row_words, int32_t* first_col,
                                     void* stream) {
  const char* fn = "speckv_expansion_mask";
  int st = check_mask(fn, mask, dtype, batch, query, columns);
  if (st) return st;
  if (batch * query == 0 || columns == 0) return SPECKV_OK;
  if (seen == nullptr) return fail(SPECKV_EINVAL, "%s: null seen positions", fn);
  st = check_current_device(fn, {mask, seen, pad, bits, first_col});
  if (st) return st;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = check_bits(fn, batch, columns, bits, row_words, first_col, s);
  if (st) return st;
  dim3 grid((unsigned)(batch * query), (unsigned)((columns + kDraftCols - 1) / kDraftCols));
  expansion_mask_kernel<<<grid, kDraftThreads, 0, s>>>(mask, dtype, query, columns, init_length, seen, seen_stride_b,
                                                       seen_stride_r, pad, pad_stride_b, pad_stride_c, err, bits,
                                                       row_words, first_col);
  return check_launch(fn);
}
