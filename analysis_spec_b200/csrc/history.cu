// Rollout-history pools (ContiguousRolloutHistory, helper/opd_history.py:10-67) and the
// accepted-feature gather of the verify round (helper/opd_generate.py:567-579).
//
// speckv_history_append moves, for up to four fields in one launch,
//   pool_f[owners[i]][start_f + w] = src_f[src_rows[i]][index_f[i][w]]     (i < n, w < width_f)
// (index_f NULL: position w; src_rows NULL: row i) and optionally writes the same
// elements to a contiguous (n, width_f, row_bytes_f) `gathered_f`. That covers the
// per-field index_copy_ of append (:24-42), the repeated initial copy of __init__
// (:12-22, src_rows = i / repeats), the history copy of a capacity grow (:34-38) and
// the gather of the accepted target features fused with their append (the gathered
// copy is the next draft step's input). One thread per element vector; each field
// uses the widest vector (16/8/4/2/1 bytes) its pointers, strides and row size allow.
//
// speckv_history_pack concatenates the used prefix of every pool row,
// dst[offsets[r] + p] = pool[r][p] for p < offsets[r + 1] - offsets[r], the single
// gather of finalize (:44-67).
#include "common.cuh"

namespace speckv {
namespace {

constexpr int kHistThreads = 256;

struct HistField {
  uint8_t* pool;
  long long pool_row, pool_pos;  // bytes
  const uint8_t* src;
  long long src_row, src_pos;    // bytes
  const int64_t* index;
  long long index_row, index_pos;  // elements
  uint8_t* gathered;
  long long row_bytes, src_positions, start, width;
  long long per_pos;  // vectors per position
  long long first;    // items of the fields before this one
  int vec;
};

struct HistTable {
  HistField f[SPECKV_HISTORY_MAX_FIELDS];
  int count;
  long long total;
};

template <int V>
__device__ __forceinline__ void move_vec(const uint8_t* s, uint8_t* d, uint8_t* g) {
  typedef typename Vec<V>::T T;
  const T x = *reinterpret_cast<const T*>(s);
  if (d != nullptr) *reinterpret_cast<T*>(d) = x;
  if (g != nullptr) *reinterpret_cast<T*>(g) = x;
}

__global__ void __launch_bounds__(kHistThreads) history_append_kernel(const HistTable t,
                                                                      const int64_t* __restrict__ owners,
                                                                      const int64_t* __restrict__ src_rows,
                                                                      long long pool_rows, unsigned long long* err) {
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x; id < t.total; id += step) {
    int fi = 0;
    while (fi + 1 < t.count && id >= t.f[fi + 1].first) ++fi;
    const HistField& f = t.f[fi];
    const long long local = id - f.first;
    const long long v = local % f.per_pos;
    const long long iw = local / f.per_pos;
    const long long w = iw % f.width;
    const long long i = iw / f.width;
    const long long pos = f.index != nullptr ? f.index[i * f.index_row + w * f.index_pos] : w;
    if (pos < 0 || pos >= f.src_positions) {
      if (v == 0) record_error(err, SPECKV_DERR_HISTORY_INDEX, pos);
      continue;
    }
    const long long srow = src_rows != nullptr ? src_rows[i] : i;
    const uint8_t* sp = f.src + srow * f.src_row + pos * f.src_pos + v * f.vec;
    uint8_t* gp = f.gathered != nullptr ? f.gathered + iw * f.row_bytes + v * f.vec : nullptr;
    uint8_t* dp = nullptr;
    if (f.pool != nullptr) {
      const long long owner = owners[i];
      if (owner < 0 || owner >= pool_rows) {
        if (v == 0 && w == 0) record_error(err, SPECKV_DERR_HISTORY_INDEX, owner);
      } else {
        dp = f.pool + owner * f.pool_row + (f.start + w) * f.pool_pos + v * f.vec;
      }
    }
    switch (f.vec) {
      case 16: move_vec<16>(sp, dp, gp); break;
      case 8: move_vec<8>(sp, dp, gp); break;
      case 4: move_vec<4>(sp, dp, gp); break;
      case 2: move_vec<2>(sp, dp, gp); break;
      default: move_vec<1>(sp, dp, gp); break;
    }
  }
}

template <int V>
__global__ void __launch_bounds__(kHistThreads) history_pack_kernel(uint8_t* __restrict__ dst,
                                                                    const uint8_t* __restrict__ pool,
                                                                    long long pool_row, long long pool_pos,
                                                                    long long row_bytes,
                                                                    const int64_t* __restrict__ offsets) {
  typedef typename Vec<V>::T T;
  const long long r = blockIdx.y;
  const long long off = offsets[r];
  const long long len = offsets[r + 1] - off;
  const long long per_pos = row_bytes / V;
  const long long items = len * per_pos;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x; id < items; id += step) {
    const long long p = id / per_pos, v = id % per_pos;
    *reinterpret_cast<T*>(dst + (off + p) * row_bytes + v * V) =
        *reinterpret_cast<const T*>(pool + r * pool_row + p * pool_pos + v * V);
  }
}

int grid_for(long long items) {
  long long blocks = (items + kHistThreads - 1) / kHistThreads;
  const long long cap = 148LL * 16;
  return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace
}  // namespace speckv

using namespace speckv;

extern "C" int speckv_history_append(int32_t fields, void* const* pools, const int64_t* pool_strides,
                                     const void* const* srcs, const int64_t* src_strides,
                                     const int64_t* const* indices, const int64_t* index_strides,
                                     void* const* gathered, const int64_t* row_bytes,
                                     const int64_t* src_positions, const int64_t* starts, const int64_t* widths,
                                     const int64_t* capacities, const int64_t* owners, const int64_t* src_rows,
                                     int64_t n, int64_t pool_rows, void* stream) {
  const char* fn = "speckv_history_append";
  if (fields < 1 || fields > SPECKV_HISTORY_MAX_FIELDS)
    return fail(SPECKV_EINVAL, "%s: %d fields (1..%d)", fn, fields, SPECKV_HISTORY_MAX_FIELDS);
  if (n < 0 || pool_rows < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (!pools || !pool_strides || !srcs || !src_strides || !row_bytes || !src_positions || !starts || !widths ||
      !capacities)
    return fail(SPECKV_EINVAL, "%s: null argument array", fn);
  HistTable t;
  t.count = fields;
  t.total = 0;
  bool any_pool = false;
  for (int f = 0; f < fields; ++f) {
    HistField& h = t.f[f];
    h.pool = static_cast<uint8_t*>(pools[f]);
    h.pool_row = pool_strides[2 * f];
    h.pool_pos = pool_strides[2 * f + 1];
    h.src = static_cast<const uint8_t*>(srcs[f]);
    h.src_row = src_strides[2 * f];
    h.src_pos = src_strides[2 * f + 1];
    h.index = indices != nullptr ? indices[f] : nullptr;
    h.index_row = index_strides != nullptr ? index_strides[2 * f] : 0;
    h.index_pos = index_strides != nullptr ? index_strides[2 * f + 1] : 0;
    h.gathered = gathered != nullptr ? static_cast<uint8_t*>(gathered[f]) : nullptr;
    h.row_bytes = row_bytes[f];
    h.src_positions = src_positions[f];
    h.start = starts[f];
    h.width = widths[f];
    if (h.row_bytes < 1 || h.width < 0 || h.start < 0)
      return fail(SPECKV_EINVAL, "%s: field %d: bad row bytes / start / width", fn, f);
    if (h.pool == nullptr && h.gathered == nullptr)
      return fail(SPECKV_EINVAL, "%s: field %d has neither a pool nor a gathered output", fn, f);
    if (h.pool != nullptr && h.start + h.width > capacities[f])
      return fail(SPECKV_EINVAL, "%s: field %d: positions %lld..%lld beyond capacity %lld", fn, f,
                  (long long)h.start, (long long)(h.start + h.width), (long long)capacities[f]);
    if (n * h.width > 0 && (h.src == nullptr || h.src_positions < 1))
      return fail(SPECKV_EINVAL, "%s: field %d: null or empty source", fn, f);
    if (h.pool != nullptr) any_pool = true;
    const long long vals[8] = {h.row_bytes, (long long)(uintptr_t)h.src, h.src_row, h.src_pos,
                               h.pool ? (long long)(uintptr_t)h.pool : 0, h.pool ? h.pool_row : 0,
                               h.pool ? h.pool_pos : 0, h.gathered ? (long long)(uintptr_t)h.gathered : 0};
    h.vec = pick_vec(vals, 8);
    h.per_pos = h.row_bytes / h.vec;
    h.first = t.total;
    t.total += n * h.width * h.per_pos;
  }
  if (t.total == 0) return SPECKV_OK;
  if (any_pool && owners == nullptr) return fail(SPECKV_EINVAL, "%s: null owners", fn);
  const int dst = check_current_device(fn, {t.f[0].src, t.f[0].pool, t.f[0].gathered, owners});
  if (dst) return dst;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  history_append_kernel<<<grid_for(t.total), kHistThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      t, owners, src_rows, pool_rows, err);
  return check_launch(fn);
}

extern "C" int speckv_history_pack(void* dst, const void* pool, int64_t pool_row_stride, int64_t pool_pos_stride,
                                   int64_t row_bytes, const int64_t* offsets, int64_t rows, int64_t max_length,
                                   void* stream) {
  const char* fn = "speckv_history_pack";
  if (rows < 0 || max_length < 0 || row_bytes < 1) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (rows == 0 || max_length == 0) return SPECKV_OK;
  if (!dst || !pool || !offsets) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (rows > 65535) return fail(SPECKV_ENOSUPPORT, "%s: more than 65535 rows", fn);
  const int dst_ok = check_current_device(fn, {dst, pool, offsets});
  if (dst_ok) return dst_ok;
  const long long vals[5] = {row_bytes, pool_row_stride, pool_pos_stride, (long long)(uintptr_t)dst,
                             (long long)(uintptr_t)pool};
  const int vec = pick_vec(vals, 5);
  const long long per_row = max_length * (row_bytes / vec);
  long long bx = (per_row + kHistThreads - 1) / kHistThreads;
  if (bx > 64) bx = 64;
  dim3 grid((unsigned)bx, (unsigned)rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* d = static_cast<uint8_t*>(dst);
  const uint8_t* p = static_cast<const uint8_t*>(pool);
  SPECKV_DISPATCH_VEC(vec, (history_pack_kernel<V><<<grid, kHistThreads, 0, s>>>(d, p, pool_row_stride,
                                                                                 pool_pos_stride, row_bytes, offsets)));
  return check_launch(fn);
}
