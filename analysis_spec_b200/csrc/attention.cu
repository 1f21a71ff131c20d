// C-ABI entries of the tree-verify attention: validate arguments and pick the
// kernel for the shape. Head dim 128 in bf16 / fp16 (every verify and draft
// attention of the Qwen2.5 geometries) runs only on the tcgen05 kernels; a view
// of that shape they cannot read (a base or stride that is not 16-byte aligned)
// is refused with SPECKV_ENOSUPPORT instead of silently taking a slower path.
// The CUDA-core kernel serves the other head dims and fp32. Both paths count
// their launches (speckv_attention_launches).
#include "common.cuh"
#include "attention.cuh"

#include <atomic>

using namespace speckv;

namespace {

std::atomic<long long> g_tensor_core_launches{0}, g_cuda_core_launches{0};

int check(const char* fn, const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
          const int64_t* vs, const void* out, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t rows,
          int64_t kv_len, int64_t dim) {
  if (batch < 0 || q_heads < 1 || kv_heads < 1 || rows < 0 || kv_len < 0 || dim < 1)
    return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (q_heads % kv_heads != 0)
    return fail(SPECKV_EINVAL, "%s: %lld query heads not a multiple of %lld kv heads", fn, (long long)q_heads,
                (long long)kv_heads);
  if (batch == 0 || rows == 0) return SPECKV_OK;
  if (kv_len == 0) return fail(SPECKV_EINVAL, "%s: empty key/value sequence", fn);
  if (!q || !k || !v || !out || !qs || !ks || !vs) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  return SPECKV_OK;
}

void fill(AttnArgs& a, const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
          const int64_t* vs, void* out, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t rows,
          int64_t kv_len, int64_t dim, float scale, int32_t dtype) {
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = qs[i];
    a.ks[i] = ks[i];
    a.vs[i] = vs[i];
  }
  a.batch = batch;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.rows = rows;
  a.kv_len = kv_len;
  a.dim = dim;
  a.scale = scale;
  a.dtype = dtype;
  a.mask = nullptr;
  a.mask_dtype = SPECKV_F32;
  a.bits = nullptr;
  a.row_words = 0;
  a.first_col = nullptr;
  a.row_table = nullptr;
  a.kv_batch = batch;
  a.past = -1;
  a.k_new = nullptr;
  a.v_new = nullptr;
  for (int i = 0; i < 3; ++i) a.kns[i] = a.vns[i] = 0;
}

int launch(const char* fn, const AttnArgs& a, cudaStream_t s) {
  int st = check_current_device(fn, {a.q, a.k, a.out, a.mask != nullptr ? a.mask : a.bits});
  if (st) return st;
  const bool tensor_shape = a.dim == 128 && (a.dtype == SPECKV_BF16 || a.dtype == SPECKV_F16);
  if (tensor_shape) {
    if (!sm100_supported(a))
      return fail(SPECKV_ENOSUPPORT,
                  "%s: head dim 128 in bf16 / fp16 runs on the tensor-core kernel only, which needs 16-byte aligned "
                  "Q / K / V / output bases and strides (and visibility rows of a multiple of 4 words), batch <= "
                  "2^20 and kv_len <= 2^30; this view does not qualify", fn);
    st = attention_sm100(a, s);
    if (st == SPECKV_OK) ++g_tensor_core_launches;
    return st;
  }
  st = attention_generic(a, s);
  if (st == SPECKV_OK) ++g_cuda_core_launches;
  return st;
}

}  // namespace

extern "C" int speckv_tree_attention(const void* q, const int64_t* q_strides,
                                     const void* k, const int64_t* k_strides,
                                     const void* v, const int64_t* v_strides,
                                     const void* mask, int32_t mask_dtype,
                                     void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                     int64_t rows, int64_t kv_len, int64_t dim, float scale,
                                     int32_t dtype, void* stream) {
  const char* fn = "speckv_tree_attention";
  int st = check(fn, q, q_strides, k, k_strides, v, v_strides, out, batch, q_heads, kv_heads, rows, kv_len, dim);
  if (st || batch == 0 || rows == 0) return st;
  if (mask != nullptr && mask_dtype != SPECKV_F32 && mask_dtype != SPECKV_BF16 && mask_dtype != SPECKV_F16)
    return fail(SPECKV_EINVAL, "%s: unsupported mask dtype %d", fn, mask_dtype);
  AttnArgs a;
  fill(a, q, q_strides, k, k_strides, v, v_strides, out, batch, q_heads, kv_heads, rows, kv_len, dim, scale, dtype);
  a.mask = mask;
  a.mask_dtype = mask_dtype;
  return launch(fn, a, static_cast<cudaStream_t>(stream));
}

extern "C" int speckv_tree_attention_bits(const void* q, const int64_t* q_strides,
                                          const void* k, const int64_t* k_strides,
                                          const void* v, const int64_t* v_strides,
                                          const uint32_t* bits, int64_t row_words, const int32_t* first_col,
                                          void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                          int64_t rows, int64_t kv_len, int64_t dim, float scale,
                                          int32_t dtype, const int64_t* row_table, int64_t kv_batch,
                                          void* stream) {
  const char* fn = "speckv_tree_attention_bits";
  int st = check(fn, q, q_strides, k, k_strides, v, v_strides, out, batch, q_heads, kv_heads, rows, kv_len, dim);
  if (st || batch == 0 || rows == 0) return st;
  if (bits == nullptr) return fail(SPECKV_EINVAL, "%s: null visibility bits", fn);
  if (row_words < 4 * ((kv_len + 127) / 128))
    return fail(SPECKV_EINVAL, "%s: row_words %lld below 4 * ceil(kv_len / 128)", fn, (long long)row_words);
  AttnArgs a;
  fill(a, q, q_strides, k, k_strides, v, v_strides, out, batch, q_heads, kv_heads, rows, kv_len, dim, scale, dtype);
  a.bits = bits;
  a.row_words = row_words;
  a.first_col = first_col;
  if (row_table != nullptr) {
    if (kv_batch < 1 || kv_batch > (1 << 20))
      return fail(SPECKV_EINVAL, "%s: row table needs the K/V row count (got %lld)", fn, (long long)kv_batch);
    a.row_table = row_table;
    a.kv_batch = kv_batch;
    if (!sm100_supported(a))
      return fail(SPECKV_ENOSUPPORT, "%s: row tables need the tensor-core path (head dim 128, bf16 / fp16, "
                  "16-byte aligned rows)", fn);
  }
  return launch(fn, a, static_cast<cudaStream_t>(stream));
}

// The round's append fused into the verify attention: the same pools and output as
// speckv_append_rows(k_new / v_new at position past, this layer) followed by
// speckv_tree_attention_bits over the past + rows positions, in one launch.
extern "C" int speckv_tree_attention_bits_append(const void* q, const int64_t* q_strides,
                                                 void* k_pool, const int64_t* k_pool_strides,
                                                 void* v_pool, const int64_t* v_pool_strides,
                                                 int64_t past, int64_t capacity,
                                                 const void* k_new, const int64_t* k_new_strides,
                                                 const void* v_new, const int64_t* v_new_strides,
                                                 const uint32_t* bits, int64_t row_words, const int32_t* first_col,
                                                 void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                                 int64_t rows, int64_t dim, float scale, int32_t dtype,
                                                 void* stream) {
  const char* fn = "speckv_tree_attention_bits_append";
  if (past < 0 || rows < 0 || capacity < 0 || past > capacity - rows)
    return fail(SPECKV_EINVAL, "%s: past %lld + rows %lld exceed the pools' %lld positions", fn, (long long)past,
                (long long)rows, (long long)capacity);
  int st = check(fn, q, q_strides, k_pool, k_pool_strides, v_pool, v_pool_strides, out, batch, q_heads, kv_heads,
                 rows, past + rows, dim);
  if (st || batch == 0 || rows == 0) return st;
  if (k_new == nullptr || v_new == nullptr || k_new_strides == nullptr || v_new_strides == nullptr)
    return fail(SPECKV_EINVAL, "%s: null new rows", fn);
  if (bits == nullptr) return fail(SPECKV_EINVAL, "%s: null visibility bits", fn);
  const int64_t kv_len = past + rows;
  if (row_words < 4 * ((kv_len + 127) / 128))
    return fail(SPECKV_EINVAL, "%s: row_words %lld below 4 * ceil(kv_len / 128)", fn, (long long)row_words);
  if (dim != 128 || (dtype != SPECKV_BF16 && dtype != SPECKV_F16))
    return fail(SPECKV_ENOSUPPORT, "%s: head dim 128 in bf16 / fp16 only", fn);
  if (rows > 128)
    return fail(SPECKV_ENOSUPPORT, "%s: %lld new rows (one 128-key tile at most)", fn, (long long)rows);
  st = check_current_device(fn, {k_new, v_new, v_pool});
  if (st) return st;
  AttnArgs a;
  fill(a, q, q_strides, k_pool, k_pool_strides, v_pool, v_pool_strides, out, batch, q_heads, kv_heads, rows, kv_len,
       dim, scale, dtype);
  a.bits = bits;
  a.row_words = row_words;
  a.first_col = first_col;
  a.past = past;
  a.k_new = k_new;
  a.v_new = v_new;
  for (int i = 0; i < 3; ++i) {
    a.kns[i] = k_new_strides[i];
    a.vns[i] = v_new_strides[i];
  }
  return launch(fn, a, static_cast<cudaStream_t>(stream));
}

extern "C" int speckv_attention_launches(int64_t* tensor_core, int64_t* cuda_core) {
  if (tensor_core == nullptr || cuda_core == nullptr)
    return fail(SPECKV_EINVAL, "speckv_attention_launches: null output");
  *tensor_core = g_tensor_core_launches.load();
  *cuda_core = g_cuda_core_launches.load();
  return SPECKV_OK;
}

extern "C" int speckv_attention_set_ctas(int32_t ctas) {
  if (ctas < 0) return fail(SPECKV_EINVAL, "speckv_attention_set_ctas: negative CTA count");
  attention_set_ctas(ctas);
  return SPECKV_OK;
}

extern "C" int speckv_attention_set_chunks(int32_t on) {
  if (on < 0 || on > 1) return fail(SPECKV_EINVAL, "speckv_attention_set_chunks: 0 or 1 expected");
  attention_set_chunks(on);
  return SPECKV_OK;
}

extern "C" int speckv_attention_test_hooks(int64_t wait_limit_ns, int32_t withhold_q_arrival) {
  if (wait_limit_ns < 0 || withhold_q_arrival < 0 || withhold_q_arrival > 1)
    return fail(SPECKV_EINVAL, "speckv_attention_test_hooks: wait limit >= 0 and a 0 / 1 switch expected");
  return attention_test_hooks(wait_limit_ns, withhold_q_arrival);
}
