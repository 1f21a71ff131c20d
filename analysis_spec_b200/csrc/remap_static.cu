// Batch remap of the KV pools for callers that cannot allocate device memory.
//
// speckv_remap_rows needs caller-provided scratch when the rows of one
// position do not fit on chip. Some callers cannot hand it any: a host that has
// given all device memory to its own pooling allocator up front (so a raw
// cudaMalloc would fail), a latency-critical loop where cudaMalloc / cudaFree
// would synchronise the device, or a foreign-language binding with no access
// to the framework's allocator. speckv_remap_rows_static does the same remap
// through a fixed scratch array compiled into this file instead.
//
// The array is a file-scope __device__ array of SPECKV_REMAP_STATIC_SCRATCH_BYTES:
// every GPU that loads this part of the library holds it until the process
// exits. Host code cannot use the array's name as a device address; the
// device address is looked up once per device with cudaGetSymbolAddress (with
// that device current) and passed to the kernels.
#include "common.cuh"

#include <mutex>

namespace speckv {
namespace {

static __device__ __align__(256) unsigned char g_remap_scratch[SPECKV_REMAP_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
constexpr int kThreads = 256;
unsigned char* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mutex;

// Device address of g_remap_scratch on the current device (looked up on first use).
int scratch_address(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SPECKV_ECUDA, "speckv_remap_rows_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(SPECKV_ENOSUPPORT, "speckv_remap_rows_static: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_remap_scratch);
    if (e != cudaSuccess)
      return fail(SPECKV_ECUDA, "speckv_remap_rows_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_ptr[dev];
  return SPECKV_OK;
}

// Positions [t0, t0 + span) of every row: gather (pass 0) into the scratch,
// then scatter (pass 1) to rows [0, new_batch).
struct ChunkGeom {
  long long sb, sh, row_bytes, nvec, t0, span, heads, new_batch, batch_cap;
  long long per_tensor;  // new_batch * heads * span * nvec vectors
};

template <int V>
__global__ void __launch_bounds__(kThreads) chunk_gather(const char* kpool, const char* vpool,
                                                         const int64_t* __restrict__ indices, char* scratch,
                                                         ChunkGeom g, unsigned long long* err) {
  typedef typename Vec<V>::T T;
  const int kv = blockIdx.y;
  const char* base = kv ? vpool : kpool;
  T* out = reinterpret_cast<T*>(scratch) + (long long)kv * g.per_tensor;
  for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < g.per_tensor;
       i += (long long)gridDim.x * kThreads) {
    const long long lv = i % g.nvec;
    const long long row = i / g.nvec;
    const long long t = row % g.span;
    const long long rh = row / g.span;
    const long long h = rh % g.heads;
    const long long r = rh / g.heads;
    const long long s = indices[r];
    if (s < 0 || s >= g.batch_cap) {
      if (lv == 0 && t == 0) record_error(err, SPECKV_DERR_REMAP_INDEX, s);
      continue;
    }
    out[i] = *reinterpret_cast<const T*>(base + s * g.sb + h * g.sh + (g.t0 + t) * g.row_bytes + lv * V);
  }
}

template <int V>
__global__ void __launch_bounds__(kThreads) chunk_scatter(char* kpool, char* vpool, const int64_t* __restrict__ indices,
                                                          const char* scratch, ChunkGeom g) {
  typedef typename Vec<V>::T T;
  const int kv = blockIdx.y;
  char* base = kv ? vpool : kpool;
  const T* in = reinterpret_cast<const T*>(scratch) + (long long)kv * g.per_tensor;
  for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < g.per_tensor;
       i += (long long)gridDim.x * kThreads) {
    const long long lv = i % g.nvec;
    const long long row = i / g.nvec;
    const long long t = row % g.span;
    const long long rh = row / g.span;
    const long long h = rh % g.heads;
    const long long r = rh / g.heads;
    const long long s = indices[r];
    if (s < 0 || s >= g.batch_cap) continue;
    *reinterpret_cast<T*>(base + r * g.sb + h * g.sh + (g.t0 + t) * g.row_bytes + lv * V) = in[i];
  }
}

}  // namespace
}  // namespace speckv

using namespace speckv;

extern "C" int speckv_remap_rows_static(void* const* key_pools, void* const* value_pools, int32_t layers,
                                        const int64_t* indices, int64_t new_batch, int64_t batch_capacity,
                                        int64_t heads, int64_t dim, int64_t capacity, int64_t length,
                                        int32_t elem_bytes, void* stream) {
  const char* fn = "speckv_remap_rows_static";
  if (layers < 1 || layers > SPECKV_MAX_LAYERS)
    return fail(SPECKV_EINVAL, "%s: layers=%d outside [1, %d]", fn, layers, SPECKV_MAX_LAYERS);
  if (key_pools == nullptr || value_pools == nullptr) return fail(SPECKV_EINVAL, "%s: null pool table", fn);
  for (int l = 0; l < layers; ++l)
    if (key_pools[l] == nullptr || value_pools[l] == nullptr) return fail(SPECKV_EINVAL, "%s: null pool for layer %d", fn, l);
  if (heads < 1 || dim < 1 || capacity < 1) return fail(SPECKV_EINVAL, "%s: heads/dim/capacity must be positive", fn);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(SPECKV_EINVAL, "%s: elem_bytes=%d unsupported", fn, elem_bytes);
  if (new_batch < 0 || length < 0 || batch_capacity < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (new_batch > batch_capacity)
    return fail(SPECKV_EINVAL, "%s: new batch %lld exceeds batch capacity %lld", fn, (long long)new_batch,
                (long long)batch_capacity);
  if (length > capacity) return fail(SPECKV_EINVAL, "%s: length exceeds capacity", fn);
  // Every size below stays under 2^31, so the byte products that follow cannot overflow
  // (an overflowed product could pass the scratch check and give a chunk <= 0).
  if (!fits_u31(new_batch) || !fits_u31(batch_capacity) || !fits_u31(heads) || !fits_u31(dim) ||
      !fits_u31(capacity) || !fits_u31(length) || !fits_u31(dim * elem_bytes))
    return fail(SPECKV_EINVAL, "%s: a size is 2^31 or more", fn);
  const long long row_bytes = dim * elem_bytes;
  // K and V rows of one position for every output row must fit; longer prefixes
  // are processed in position chunks. Compared by division first, so that the
  // product below is only formed once it is known to fit.
  const long long rows_fit = (long long)SPECKV_REMAP_STATIC_SCRATCH_BYTES / (2 * row_bytes);
  if (new_batch > 0 && heads > rows_fit / new_batch)
    return fail(SPECKV_EINVAL,
                "%s: %lld rows x %lld heads x %lld-byte rows (K and V) exceed the %lld-byte static scratch per "
                "position; use speckv_remap_rows with caller scratch",
                fn, (long long)new_batch, (long long)heads, row_bytes, (long long)SPECKV_REMAP_STATIC_SCRATCH_BYTES);
  const long long per_position = 2 * new_batch * heads * row_bytes;
  if (new_batch == 0 || length == 0) return SPECKV_OK;
  if (indices == nullptr) return fail(SPECKV_EINVAL, "%s: null indices", fn);
  int st = check_current_device(fn, {key_pools[0], value_pools[0], indices});
  if (st) return st;
  unsigned char* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st) return st;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  long long vals[2 * SPECKV_MAX_LAYERS + 1];
  int nv = 0;
  vals[nv++] = row_bytes;
  for (int l = 0; l < layers; ++l) {
    vals[nv++] = (long long)(uintptr_t)key_pools[l];
    vals[nv++] = (long long)(uintptr_t)value_pools[l];
  }
  const int vec = pick_vec(vals, nv);
  const long long chunk = (long long)SPECKV_REMAP_STATIC_SCRATCH_BYTES / per_position;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int l = 0; l < layers; ++l) {
    char* kp = static_cast<char*>(key_pools[l]);
    char* vp = static_cast<char*>(value_pools[l]);
    for (long long t0 = 0; t0 < length; t0 += chunk) {
      ChunkGeom g;
      g.row_bytes = row_bytes;
      g.nvec = row_bytes / vec;
      g.sh = capacity * row_bytes;
      g.sb = heads * g.sh;
      g.t0 = t0;
      g.span = (length - t0) < chunk ? (length - t0) : chunk;
      g.heads = heads;
      g.new_batch = new_batch;
      g.batch_cap = batch_capacity;
      g.per_tensor = new_batch * heads * g.span * g.nvec;
      long long blocks = (g.per_tensor + kThreads - 1) / kThreads;
      if (blocks > 148 * 16) blocks = 148 * 16;
      dim3 grid((unsigned)blocks, 2);
      char* scr = reinterpret_cast<char*>(scratch);
      SPECKV_DISPATCH_VEC(vec, {
        chunk_gather<V><<<grid, kThreads, 0, s>>>(kp, vp, indices, scr, g, err);
        chunk_scatter<V><<<grid, kThreads, 0, s>>>(kp, vp, indices, scr, g);
      });
      st = check_launch(fn);
      if (st) return st;
    }
  }
  return SPECKV_OK;
}
