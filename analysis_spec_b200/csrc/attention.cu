// C-ABI entry of the tree-verify attention: validates arguments and picks the
// kernel for the shape.
#include "common.cuh"
#include "attention.cuh"

using namespace speckv;

extern "C" int speckv_tree_attention(const void* q, const int64_t* q_strides,
                                     const void* k, const int64_t* k_strides,
                                     const void* v, const int64_t* v_strides,
                                     const void* mask, int32_t mask_dtype,
                                     void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                     int64_t rows, int64_t kv_len, int64_t dim, float scale,
                                     int32_t dtype, void* stream) {
  const char* fn = "speckv_tree_attention";
  if (batch < 0 || q_heads < 1 || kv_heads < 1 || rows < 0 || kv_len < 0 || dim < 1)
    return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (q_heads % kv_heads != 0)
    return fail(SPECKV_EINVAL, "%s: %lld query heads not a multiple of %lld kv heads", fn, (long long)q_heads,
                (long long)kv_heads);
  if (batch == 0 || rows == 0) return SPECKV_OK;
  if (kv_len == 0) return fail(SPECKV_EINVAL, "%s: empty key/value sequence", fn);
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (mask != nullptr && mask_dtype != SPECKV_F32 && mask_dtype != SPECKV_BF16 && mask_dtype != SPECKV_F16)
    return fail(SPECKV_EINVAL, "%s: unsupported mask dtype %d", fn, mask_dtype);
  AttnArgs a;
  a.q = q; a.k = k; a.v = v; a.mask = mask; a.out = out;
  for (int i = 0; i < 3; ++i) { a.qs[i] = q_strides[i]; a.ks[i] = k_strides[i]; a.vs[i] = v_strides[i]; }
  a.batch = batch; a.q_heads = q_heads; a.kv_heads = kv_heads; a.rows = rows; a.kv_len = kv_len; a.dim = dim;
  a.scale = scale; a.dtype = dtype; a.mask_dtype = mask_dtype;
  return attention_generic(a, static_cast<cudaStream_t>(stream));
}
