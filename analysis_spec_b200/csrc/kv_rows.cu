// KV row movement kernels of the static cache: append, accepted-suffix
// compaction, batch remap and tail-to-hole release. Every kernel is a
// vectorised (up to 16-byte) copy of whole (sequence, head, position) rows of
// the per-layer pools, and every kernel covers all layers and both K and V in
// one launch (blockIdx.y / the group index selects layer * 2 + kv).
//
// These replace the reference's per-layer torch copy_/gather calls and Triton
// kernels (helper/opd_static_cache.py:99-174, helper/opd_kv_kernels.py:11-58,
// helper/opd_scheduling.py:35-58); results are byte-identical.
#include "common.cuh"
#include "positions.cuh"

#include <limits.h>

namespace speckv {
namespace {

constexpr int kThreads = 256;

struct PoolTable {
  char* ptr[2 * SPECKV_MAX_LAYERS];  // index = layer * 2 + kv
};
struct SrcTable {
  const char* ptr[2 * SPECKV_MAX_LAYERS];
};

// Optional logical -> physical pool row table: logical sequence b lives in pool row map[b]
// (NULL: row b). An entry outside [0, rows) is reported in the device error word and that
// sequence is skipped, so a bad table never addresses memory outside the pools.
struct RowTable {
  const int64_t* map;
  long long rows;
};
__device__ __forceinline__ long long phys_row(const RowTable& t, long long b, unsigned long long* err) {
  if (t.map == nullptr) return b;
  const long long p = t.map[b];
  if (p < 0 || p >= t.rows) {
    record_error(err, SPECKV_DERR_ROW_TABLE, p);
    return -1;
  }
  return p;
}

template <int V>
__device__ __forceinline__ typename Vec<V>::T load_vec(const char* p) {
  return *reinterpret_cast<const typename Vec<V>::T*>(p);
}
template <int V>
__device__ __forceinline__ void store_vec(char* p, typename Vec<V>::T x) {
  *reinterpret_cast<typename Vec<V>::T*>(p) = x;
}

// ---------------------------------------------------------------------------
// append: pool[b][h][t0 + t] = src[b][h][t] for all (b, h, t)
// ---------------------------------------------------------------------------
struct AppendGeom {
  FastDiv nvec;   // vectors per row
  FastDiv rows;   // appended positions per (b, h)
  FastDiv heads;  // heads
  long long dst_sb, dst_sh, dst_t0, row_bytes;
  long long src_sb[2], src_sh[2], src_st[2];  // byte strides of the K / V source
  uint32_t total;                             // vectors per tensor
  RowTable rt;                                // destination pool row of each sequence
  unsigned long long* err;
};

template <int V, int UNROLL>
__global__ void __launch_bounds__(kThreads) append_kernel(PoolTable dst, SrcTable src, AppendGeom g) {
  typedef typename Vec<V>::T T;
  const int tensor = blockIdx.y;
  const int kv = tensor & 1;
  char* __restrict__ d = dst.ptr[tensor];
  const char* __restrict__ s = src.ptr[tensor];
  const uint32_t base = blockIdx.x * (kThreads * UNROLL) + threadIdx.x;
  T buf[UNROLL];
  long long doff[UNROLL];
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    const uint32_t i = base + u * kThreads;
    doff[u] = -1;
    if (i < g.total) {
      uint32_t row, lane, bh, t, b, h;
      g.nvec.divmod(i, row, lane);
      g.rows.divmod(row, bh, t);
      g.heads.divmod(bh, b, h);
      const long long pb = phys_row(g.rt, b, g.err);
      if (pb >= 0) {
        const long long so = (long long)b * g.src_sb[kv] + (long long)h * g.src_sh[kv] +
                             (long long)t * g.src_st[kv] + (long long)lane * V;
        buf[u] = load_vec<V>(s + so);
        doff[u] = pb * g.dst_sb + (long long)h * g.dst_sh + g.dst_t0 + (long long)t * g.row_bytes +
                  (long long)lane * V;
      }
    }
  }
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    if (doff[u] >= 0) store_vec<V>(d + doff[u], buf[u]);
  }
}

// ---------------------------------------------------------------------------
// compact: per (tensor, b, h) group, gather rows chosen[b][e + j] then write
// them to past + e + j. One warp per group, rows staged in registers.
// ---------------------------------------------------------------------------
struct CompactGeom {
  FastDiv bh;     // batch * heads
  FastDiv heads;  // heads
  FastDiv nvec;   // vectors per row
  long long sb, sh, row_bytes;
  long long length, past, extension;
  long long csb, csw;  // chosen strides (elements)
  uint32_t n;          // rows per group (width - extension)
  uint32_t groups;     // 2 * layers * batch * heads
  RowTable rt;         // pool row of each sequence
};

template <int V, int MAXR>
__global__ void __launch_bounds__(kThreads) compact_warp_kernel(PoolTable pools, const int64_t* __restrict__ chosen,
                                                                CompactGeom g, unsigned long long* err) {
  typedef typename Vec<V>::T T;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t group = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  if (group >= g.groups) return;
  uint32_t tensor, bh, b, h;
  g.bh.divmod(group, tensor, bh);
  g.heads.divmod(bh, b, h);
  const long long pb = phys_row(g.rt, b, err);
  if (pb < 0) return;  // the whole warp shares b
  char* base = pools.ptr[tensor] + pb * g.sb + (long long)h * g.sh;
  const uint32_t nv = g.n * g.nvec.d;
  T buf[MAXR];
  long long src[MAXR];
#pragma unroll
  for (int r = 0; r < MAXR; ++r) {
    const uint32_t i = lane + r * 32;
    src[r] = -1;
    if (i < nv) {
      uint32_t j, lv;
      g.nvec.divmod(i, j, lv);
      const long long pos = chosen[(long long)b * g.csb + (g.extension + j) * g.csw];
      if (pos < 0 || pos >= g.length) {
        record_error(err, SPECKV_DERR_COMPACT_INDEX, pos);
      } else {
        src[r] = pos;
        buf[r] = load_vec<V>(base + pos * g.row_bytes + (long long)lv * V);
      }
    }
  }
  __syncwarp();
#pragma unroll
  for (int r = 0; r < MAXR; ++r) {
    const uint32_t i = lane + r * 32;
    if (i < nv && src[r] >= 0) {
      uint32_t j, lv;
      g.nvec.divmod(i, j, lv);
      store_vec<V>(base + (g.past + g.extension + j) * g.row_bytes + (long long)lv * V, buf[r]);
    }
  }
}

// Same contract with the group staged in shared memory (one CTA per group),
// for groups larger than the register stage.
template <int V>
__global__ void __launch_bounds__(kThreads) compact_smem_kernel(PoolTable pools, const int64_t* __restrict__ chosen,
                                                                CompactGeom g, unsigned long long* err) {
  typedef typename Vec<V>::T T;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* stage = reinterpret_cast<T*>(smem_raw);
  const uint32_t group = blockIdx.x;
  uint32_t tensor, bh, b, h;
  g.bh.divmod(group, tensor, bh);
  g.heads.divmod(bh, b, h);
  const long long pb = phys_row(g.rt, b, err);
  if (pb < 0) return;  // the whole CTA shares b
  char* base = pools.ptr[tensor] + pb * g.sb + (long long)h * g.sh;
  const uint32_t nv = g.n * g.nvec.d;
  for (uint32_t i = threadIdx.x; i < nv; i += kThreads) {
    uint32_t j, lv;
    g.nvec.divmod(i, j, lv);
    const long long pos = chosen[(long long)b * g.csb + (g.extension + j) * g.csw];
    if (pos >= 0 && pos < g.length) stage[i] = load_vec<V>(base + pos * g.row_bytes + (long long)lv * V);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < nv; i += kThreads) {
    uint32_t j, lv;
    g.nvec.divmod(i, j, lv);
    const long long pos = chosen[(long long)b * g.csb + (g.extension + j) * g.csw];
    if (pos < 0 || pos >= g.length) {
      if (lv == 0) record_error(err, SPECKV_DERR_COMPACT_INDEX, pos);
      continue;
    }
    store_vec<V>(base + (g.past + g.extension + j) * g.row_bytes + (long long)lv * V, stage[i]);
  }
}

// ---------------------------------------------------------------------------
// remap, single pass: a CTA owns positions [t0, t0 + tile) of one head of one
// tensor for ALL batch rows, so it can read every source row into shared
// memory before writing any destination row; CTAs touch disjoint columns.
// ---------------------------------------------------------------------------
struct RemapGeom {
  FastDiv row_vecs;  // tile * nvec: vectors per batch row inside a CTA
  FastDiv nvec;
  FastDiv tiles;     // position tiles per head
  long long sb, sh, row_bytes;
  uint32_t new_batch, batch_cap, tile, length;
};

template <int V>
__global__ void __launch_bounds__(kThreads) remap_smem_kernel(PoolTable pools, const int64_t* __restrict__ indices,
                                                              RemapGeom g, unsigned long long* err) {
  typedef typename Vec<V>::T T;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* stage = reinterpret_cast<T*>(smem_raw);
  uint32_t h, tile_id;
  g.tiles.divmod(blockIdx.x, h, tile_id);
  const uint32_t t0 = tile_id * g.tile;
  const uint32_t tile_len = min(g.tile, g.length - t0);
  char* base = pools.ptr[blockIdx.y] + (long long)h * g.sh + (long long)t0 * g.row_bytes;
  const uint32_t total = g.new_batch * g.row_vecs.d;
  for (uint32_t i = threadIdx.x; i < total; i += kThreads) {
    uint32_t row, rem, tt, lv;
    g.row_vecs.divmod(i, row, rem);
    g.nvec.divmod(rem, tt, lv);
    if (tt >= tile_len) continue;
    const long long s = indices[row];
    if (s < 0 || s >= (long long)g.batch_cap) continue;
    stage[i] = load_vec<V>(base + s * g.sb + (long long)tt * g.row_bytes + (long long)lv * V);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < total; i += kThreads) {
    uint32_t row, rem, tt, lv;
    g.row_vecs.divmod(i, row, rem);
    g.nvec.divmod(rem, tt, lv);
    if (tt >= tile_len) continue;
    const long long s = indices[row];
    if (s < 0 || s >= (long long)g.batch_cap) {
      if (rem == 0) record_error(err, SPECKV_DERR_REMAP_INDEX, s);
      continue;
    }
    store_vec<V>(base + (long long)row * g.sb + (long long)tt * g.row_bytes + (long long)lv * V, stage[i]);
  }
}

// remap, two phases through caller scratch (one layer per launch pair; the
// stream order between the two launches is the read-before-write barrier).
struct RemapScratchGeom {
  long long sb, sh, row_bytes, nvec, length, heads;
  long long new_batch, batch_cap;
  long long per_tensor;  // vectors per tensor = new_batch * heads * length * nvec
};

template <int V>
__global__ void __launch_bounds__(kThreads) remap_gather_kernel(const char* kpool, const char* vpool, const int64_t* __restrict__ indices,
                                                                char* scratch, RemapScratchGeom g, unsigned long long* err) {
  const int kv = blockIdx.y;
  const char* base = kv ? vpool : kpool;
  char* out = scratch + (long long)kv * g.per_tensor * V;
  for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < g.per_tensor;
       i += (long long)gridDim.x * kThreads) {
    const long long lv = i % g.nvec;
    const long long row = i / g.nvec;  // (r, h, t) with t fastest
    const long long t = row % g.length;
    const long long rh = row / g.length;
    const long long h = rh % g.heads;
    const long long r = rh / g.heads;
    const long long s = indices[r];
    if (s < 0 || s >= g.batch_cap) {
      if (lv == 0 && t == 0) record_error(err, SPECKV_DERR_REMAP_INDEX, s);
      continue;
    }
    store_vec<V>(out + i * V, load_vec<V>(base + s * g.sb + h * g.sh + t * g.row_bytes + lv * V));
  }
}

template <int V>
__global__ void __launch_bounds__(kThreads) remap_scatter_kernel(char* kpool, char* vpool, const int64_t* __restrict__ indices,
                                                                 const char* scratch, RemapScratchGeom g) {
  const int kv = blockIdx.y;
  char* base = kv ? vpool : kpool;
  const char* in = scratch + (long long)kv * g.per_tensor * V;
  for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < g.per_tensor;
       i += (long long)gridDim.x * kThreads) {
    const long long lv = i % g.nvec;
    const long long row = i / g.nvec;
    const long long t = row % g.length;
    const long long rh = row / g.length;
    const long long h = rh % g.heads;
    const long long r = rh / g.heads;
    const long long s = indices[r];
    if (s < 0 || s >= g.batch_cap) continue;
    store_vec<V>(base + r * g.sb + h * g.sh + t * g.row_bytes + lv * V, load_vec<V>(in + i * V));
  }
}

// ---------------------------------------------------------------------------
// move rows: pool[dst[j]][h][0:length] = pool[src[j]][h][0:length]
// ---------------------------------------------------------------------------
struct MoveGeom {
  FastDiv span;   // length * nvec vectors per (j, h)
  FastDiv heads;
  long long sb, sh;
  uint32_t batch_cap;
  uint32_t total;  // count * heads * length * nvec
};

template <int V, int UNROLL>
__global__ void __launch_bounds__(kThreads) move_rows_kernel(PoolTable pools, const int64_t* __restrict__ sources,
                                                             const int64_t* __restrict__ dests, MoveGeom g,
                                                             unsigned long long* err) {
  typedef typename Vec<V>::T T;
  char* base = pools.ptr[blockIdx.y];
  const uint32_t first = blockIdx.x * (kThreads * UNROLL) + threadIdx.x;
  T buf[UNROLL];
  long long doff[UNROLL];
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    const uint32_t i = first + u * kThreads;
    doff[u] = -1;
    if (i < g.total) {
      uint32_t jh, off, j, h;
      g.span.divmod(i, jh, off);
      g.heads.divmod(jh, j, h);
      const long long s = sources[j];
      const long long d = dests[j];
      if (s < 0 || s >= (long long)g.batch_cap || d < 0 || d >= (long long)g.batch_cap) {
        if (off == 0) record_error(err, SPECKV_DERR_MOVE_INDEX, (s < 0 || s >= (long long)g.batch_cap) ? s : d);
        continue;
      }
      buf[u] = load_vec<V>(base + s * g.sb + (long long)h * g.sh + (long long)off * V);
      doff[u] = d * g.sb + (long long)h * g.sh + (long long)off * V;
    }
  }
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    if (doff[u] >= 0) store_vec<V>(base + doff[u], buf[u]);
  }
}

// ---------------------------------------------------------------------------
// commit round: the accepted-suffix compaction of every layer and the
// per-sequence position / padding update in one launch, with the round's width
// (longest accepted path) and extension (shortest untouched prefix over live
// sequences) reduced from the scheduling packet on the device. Nothing waits
// for the host to read the packet, so the commit runs straight after the
// packet is written.
// ---------------------------------------------------------------------------
struct RoundGeom {
  CompactGeom c;             // extension and n unused: both come from the packet
  const int64_t* chosen;     // (batch, >= max_width) cache positions of the padded paths
  const int64_t* packet;     // (batch, ps) rows [length, eos?, extension, ...]
  long long ps;
  uint32_t batch, max_width;
  uint32_t compact_blocks;   // blocks [0, compact_blocks) compact, the rest update positions
  PositionArgs pos;          // positions == null: no position update
};

// Round width and extension are reduced from the packet by warp 0 while every warp already
// loads its group's rows: the chosen positions and rows of all max_width slots are read
// speculatively (a slot outside [extension, width) is simply not stored), so the packet
// reduction, the index load and the row load are not three dependent round trips.
template <int V, int MAXR>
__global__ void __launch_bounds__(kThreads) commit_round_kernel(PoolTable pools, RoundGeom g,
                                                                unsigned long long* err) {
  typedef typename Vec<V>::T T;
  __shared__ int s_width, s_ext;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t warp = threadIdx.x >> 5;
  const bool compact = blockIdx.x < g.compact_blocks;
  const uint32_t group = blockIdx.x * (kThreads / 32) + warp;
  // speculative loads of this warp's group (compaction blocks only)
  T buf[MAXR];
  long long src[MAXR];  // source position, -1 = not loaded
  char* base = nullptr;
  uint32_t b = 0;
#pragma unroll
  for (int r = 0; r < MAXR; ++r) src[r] = -1;
  if (compact && group < g.c.groups) {
    uint32_t tensor, bh, h;
    g.c.bh.divmod(group, tensor, bh);
    g.c.heads.divmod(bh, b, h);
    const long long pb = phys_row(g.c.rt, b, err);
    if (pb >= 0) {
      base = pools.ptr[tensor] + pb * g.c.sb + (long long)h * g.c.sh;
      const uint32_t nv = g.max_width * g.c.nvec.d;
#pragma unroll
      for (int r = 0; r < MAXR; ++r) {
        const uint32_t i = lane + r * 32;
        if (i < nv) {
          uint32_t j, lv;
          g.c.nvec.divmod(i, j, lv);
          const long long pos = g.chosen[(long long)b * g.c.csb + (long long)j * g.c.csw];
          if (pos >= 0 && pos < g.c.length) {  // out of range: reported at the store if committed
            src[r] = pos;
            buf[r] = load_vec<V>(base + pos * g.c.row_bytes + (long long)lv * V);
          }
        }
      }
    }
  }
  if (warp == 0) {
    long long wmax = 0, emin = LLONG_MAX;
    for (uint32_t bb = lane; bb < g.batch; bb += 32) {
      const int64_t* row = g.packet + (long long)bb * g.ps;
      const long long len = row[0];
      wmax = len > wmax ? len : wmax;
      if (row[1] == 0 && row[2] < emin) emin = row[2];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long w2 = __shfl_xor_sync(0xffffffffu, wmax, o);
      const long long e2 = __shfl_xor_sync(0xffffffffu, emin, o);
      wmax = w2 > wmax ? w2 : wmax;
      emin = e2 < emin ? e2 : emin;
    }
    if (emin == LLONG_MAX) emin = wmax;  // no live sequence: nothing to move
    const bool ok = wmax <= g.max_width && wmax <= g.c.length - g.c.past && emin >= 0 && emin <= wmax;
    if (lane == 0) {
      if (!ok && blockIdx.x == 0) record_error(err, SPECKV_DERR_PACKET, wmax);
      s_width = ok ? (int)wmax : -1;
      s_ext = (int)emin;
    }
  }
  __syncthreads();
  const int width = s_width, ext = s_ext;
  if (width < 0) return;
  if (!compact) {
    const long long bp = (long long)(blockIdx.x - g.compact_blocks) * (kThreads / 32) + warp;
    if (bp < g.batch && width > 0) position_row(g.pos, bp, g.c.past, width, lane, err);
    return;
  }
  if (base == nullptr) return;  // beyond the groups, or a row-table entry out of range (recorded)
  // every read of this group happened above, before any write: overlapping slots are safe
#pragma unroll
  for (int r = 0; r < MAXR; ++r) {
    const uint32_t i = lane + r * 32;
    uint32_t j, lv;
    g.c.nvec.divmod(i, j, lv);
    if ((int)j < ext || (int)j >= width || i >= g.max_width * g.c.nvec.d) continue;
    if (src[r] < 0) {  // a slot of the committed range whose position is out of [0, length)
      if (lv == 0)
        record_error(err, SPECKV_DERR_COMPACT_INDEX, g.chosen[(long long)b * g.c.csb + (long long)j * g.c.csw]);
      continue;
    }
    store_vec<V>(base + (g.c.past + j) * g.c.row_bytes + (long long)lv * V, buf[r]);
  }
}

// ---------------------------------------------------------------------------
// append fused with the previous round's compaction: a round's new rows are appended in the
// same launch that moves the previous round's accepted rows chosen[b][j], j in [ext, width),
// to past + j. The compaction only has to land before the next attention reads the cache, so
// it rides on the bandwidth-bound append instead of a latency-bound launch of its own. One
// CTA per (layer, K/V, sequence, head) group reads every row it moves (the accepted rows and
// the new rows) into registers, then stores the compacted rows, then the new rows: the new
// rows may overwrite the old tree rows the accepted ones came from, and where the two
// destinations overlap (a cache cropped back below past + width) the new rows win.
// ---------------------------------------------------------------------------
constexpr int kFoldThreads = 128;
constexpr int kFoldMaxC = 2;  // compaction vectors per thread
struct FoldGeom {
  AppendGeom a;             // the append; a.dst_t0 = its first position
  FastDiv bh;               // batch * heads
  const int64_t* chosen;    // (batch, >= width) cache positions of the previous round's paths
  long long csb, csw;       // chosen strides (elements)
  long long past;           // the previous round's past: slot j goes to past + j
  long long capacity;       // accepted positions must lie in [0, capacity)
  int ext, width;           // slots [ext, width) move
  unsigned long long* err;
};

template <int V, int MAXA>
__global__ void __launch_bounds__(kFoldThreads) append_commit_kernel(PoolTable dst, SrcTable src, FoldGeom g) {
  typedef typename Vec<V>::T T;
  uint32_t tensor, bh, b, h;
  g.bh.divmod(blockIdx.x, tensor, bh);
  g.a.heads.divmod(bh, b, h);
  const int kv = tensor & 1;
  char* __restrict__ base = dst.ptr[tensor] + (long long)b * g.a.dst_sb + (long long)h * g.a.dst_sh;
  const char* __restrict__ sbase = src.ptr[tensor] + (long long)b * g.a.src_sb[kv] + (long long)h * g.a.src_sh[kv];
  const uint32_t nvec = g.a.nvec.d;
  // accepted rows of the previous round
  T cbuf[kFoldMaxC];
  long long cdst[kFoldMaxC];
  const uint32_t nc = (uint32_t)(g.width - g.ext) * nvec;
#pragma unroll
  for (int u = 0; u < kFoldMaxC; ++u) {
    const uint32_t i = threadIdx.x + u * kFoldThreads;
    cdst[u] = -1;
    if (i < nc) {
      uint32_t j, lv;
      g.a.nvec.divmod(i, j, lv);
      j += g.ext;
      const long long pos = g.chosen[(long long)b * g.csb + (long long)j * g.csw];
      if (pos >= 0 && pos < g.capacity) {
        cbuf[u] = load_vec<V>(base + pos * g.a.row_bytes + (long long)lv * V);
        cdst[u] = (g.past + j) * g.a.row_bytes + (long long)lv * V;
      } else if (lv == 0) {
        record_error(g.err, SPECKV_DERR_COMPACT_INDEX, pos);
      }
    }
  }
  // this round's new rows
  T abuf[MAXA];
  const uint32_t na = g.a.rows.d * nvec;
#pragma unroll
  for (int u = 0; u < MAXA; ++u) {
    const uint32_t i = threadIdx.x + u * kFoldThreads;
    if (i < na) {
      uint32_t t, lv;
      g.a.nvec.divmod(i, t, lv);
      abuf[u] = load_vec<V>(sbase + (long long)t * g.a.src_st[kv] + (long long)lv * V);
    }
  }
  __syncthreads();  // every row of the group is read before any is written
#pragma unroll
  for (int u = 0; u < kFoldMaxC; ++u)
    if (cdst[u] >= 0) store_vec<V>(base + cdst[u], cbuf[u]);
  __syncthreads();  // the new rows land last
#pragma unroll
  for (int u = 0; u < MAXA; ++u) {
    const uint32_t i = threadIdx.x + u * kFoldThreads;
    if (i < na) store_vec<V>(base + g.a.dst_t0 + (long long)i * V, abuf[u]);
  }
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
int check_common(const char* fn, void* const* kp, void* const* vp, int32_t layers, int64_t heads,
                 int64_t dim, int64_t capacity, int32_t elem_bytes) {
  if (layers < 1 || layers > SPECKV_MAX_LAYERS)
    return fail(SPECKV_EINVAL, "%s: layers=%d outside [1, %d]", fn, layers, SPECKV_MAX_LAYERS);
  if (kp == nullptr || vp == nullptr) return fail(SPECKV_EINVAL, "%s: null pool table", fn);
  for (int l = 0; l < layers; ++l)
    if (kp[l] == nullptr || vp[l] == nullptr) return fail(SPECKV_EINVAL, "%s: null pool for layer %d", fn, l);
  if (heads < 1 || dim < 1 || capacity < 1)
    return fail(SPECKV_EINVAL, "%s: heads/dim/capacity must be positive", fn);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(SPECKV_EINVAL, "%s: elem_bytes=%d unsupported", fn, elem_bytes);
  return SPECKV_OK;
}

void fill_pools(PoolTable& t, void* const* kp, void* const* vp, int layers) {
  for (int l = 0; l < layers; ++l) {
    t.ptr[2 * l] = static_cast<char*>(kp[l]);
    t.ptr[2 * l + 1] = static_cast<char*>(vp[l]);
  }
}

// Vector width valid for every pool base address and the row size.
int pool_vec(void* const* kp, void* const* vp, int layers, long long row_bytes) {
  long long vals[2 * SPECKV_MAX_LAYERS + 1];
  int n = 0;
  vals[n++] = row_bytes;
  for (int l = 0; l < layers; ++l) {
    vals[n++] = (long long)(uintptr_t)kp[l];
    vals[n++] = (long long)(uintptr_t)vp[l];
  }
  return pick_vec(vals, n);
}

// A validated, packed launch: host work before the enqueue is done once, at preparation.
struct LaunchPlan {
  int device = -1;  // the GPU the plan was prepared on (its pointers live there)
  virtual ~LaunchPlan() = default;
  virtual int launch(cudaStream_t s) const = 0;
};
struct EmptyPlan final : LaunchPlan {
  int launch(cudaStream_t) const override { return SPECKV_OK; }
};
struct AppendPlan final : LaunchPlan {
  PoolTable dst;
  SrcTable src;
  AppendGeom g;
  int vec;
  dim3 grid;
  int launch(cudaStream_t s) const override {
    constexpr int UNROLL = 4;
    SPECKV_DISPATCH_VEC(vec, append_kernel<V, UNROLL><<<grid, kThreads, 0, s>>>(dst, src, g));
    return check_launch("speckv_append_rows");
  }
};
struct CommitPlan final : LaunchPlan {
  PoolTable pools;
  RoundGeom g;
  unsigned long long* err;
  int vec, maxr;
  unsigned grid;
  int launch(cudaStream_t s) const override {
    if (maxr == 4) {
      SPECKV_DISPATCH_VEC(vec, commit_round_kernel<V, 4><<<grid, kThreads, 0, s>>>(pools, g, err));
    } else if (maxr == 8) {
      SPECKV_DISPATCH_VEC(vec, commit_round_kernel<V, 8><<<grid, kThreads, 0, s>>>(pools, g, err));
    } else {
      SPECKV_DISPATCH_VEC(vec, commit_round_kernel<V, 16><<<grid, kThreads, 0, s>>>(pools, g, err));
    }
    return check_launch("speckv_commit_round");
  }
};

struct FoldPlan final : LaunchPlan {
  PoolTable dst;
  SrcTable src;
  FoldGeom g;
  int vec, maxa;
  unsigned grid;
  int launch(cudaStream_t s) const override {
    if (maxa == 8) {
      SPECKV_DISPATCH_VEC(vec, append_commit_kernel<V, 8><<<grid, kFoldThreads, 0, s>>>(dst, src, g));
    } else if (maxa == 16) {
      SPECKV_DISPATCH_VEC(vec, append_commit_kernel<V, 16><<<grid, kFoldThreads, 0, s>>>(dst, src, g));
    } else {
      SPECKV_DISPATCH_VEC(vec, append_commit_kernel<V, 32><<<grid, kFoldThreads, 0, s>>>(dst, src, g));
    }
    return check_launch("speckv_append_commit_rows");
  }
};

int prepare_append(void* const* key_pools, void* const* value_pools, const void* const* key_srcs,
                   const void* const* value_srcs, int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                   int64_t dim, int64_t capacity, int64_t length, const int64_t* key_src_strides,
                   const int64_t* value_src_strides, int32_t elem_bytes, const int64_t* row_table,
                   int64_t pool_rows, LaunchPlan** out);
int prepare_fold(void* const* key_pools, void* const* value_pools, const void* const* key_srcs,
                 const void* const* value_srcs, int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                 int64_t dim, int64_t capacity, int64_t length, const int64_t* key_src_strides,
                 const int64_t* value_src_strides, int32_t elem_bytes, const int64_t* chosen,
                 int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past, int64_t extension, int64_t width,
                 LaunchPlan** out);
int prepare_commit(void* const* key_pools, void* const* value_pools, int32_t layers, int64_t batch, int64_t heads,
                   int64_t dim, int64_t capacity, int64_t length, int32_t elem_bytes, const int64_t* chosen,
                   int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past, const int64_t* packet,
                   int64_t packet_stride, int64_t max_width, uint8_t* pad_rows, int64_t pad_rows_stride,
                   int64_t pad_rows_count, const int64_t* owners, uint8_t* pad_live, int64_t pad_live_stride,
                   const uint8_t* newly_padded, int64_t np_stride_b, int64_t* positions,
                   int64_t positions_stride_b, int64_t* past_positions, const int64_t* row_table,
                   int64_t pool_rows, LaunchPlan** out);

// A row table needs the pools' row count to bound its entries.
int check_table(const char* fn, const int64_t* row_table, int64_t pool_rows, int64_t batch) {
  if (row_table != nullptr && pool_rows < 1)
    return fail(SPECKV_EINVAL, "%s: a row table needs the pools' row count", fn);
  if (row_table == nullptr && pool_rows != 0 && pool_rows < batch)
    return fail(SPECKV_EINVAL, "%s: %lld pool rows for %lld sequences", fn, (long long)pool_rows, (long long)batch);
  return SPECKV_OK;
}

// Runs a prepared plan once and frees it.
int launch_once(int st, LaunchPlan* plan, void* stream) {
  if (st) return st;
  const int r = plan->launch(static_cast<cudaStream_t>(stream));
  delete plan;
  return r;
}

}  // namespace
}  // namespace speckv

using namespace speckv;

extern "C" int speckv_append_rows(void* const* key_pools, void* const* value_pools,
                                  const void* const* key_srcs, const void* const* value_srcs,
                                  int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                                  int64_t dim, int64_t capacity, int64_t length,
                                  const int64_t* key_src_strides, const int64_t* value_src_strides,
                                  int32_t elem_bytes, const int64_t* row_table, int64_t pool_rows, void* stream) {
  LaunchPlan* plan = nullptr;
  const int st = prepare_append(key_pools, value_pools, key_srcs, value_srcs, layers, batch, heads, rows, dim,
                                capacity, length, key_src_strides, value_src_strides, elem_bytes, row_table,
                                pool_rows, &plan);
  return launch_once(st, plan, stream);
}

extern "C" int speckv_append_rows_prepare(void* const* key_pools, void* const* value_pools,
                                          const void* const* key_srcs, const void* const* value_srcs,
                                          int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                                          int64_t dim, int64_t capacity, int64_t length,
                                          const int64_t* key_src_strides, const int64_t* value_src_strides,
                                          int32_t elem_bytes, const int64_t* row_table, int64_t pool_rows,
                                          void** plan) {
  if (plan == nullptr) return fail(SPECKV_EINVAL, "speckv_append_rows_prepare: null plan");
  LaunchPlan* p = nullptr;
  const int st = prepare_append(key_pools, value_pools, key_srcs, value_srcs, layers, batch, heads, rows, dim,
                                capacity, length, key_src_strides, value_src_strides, elem_bytes, row_table,
                                pool_rows, &p);
  *plan = st ? nullptr : p;
  return st;
}

extern "C" int speckv_append_commit_rows(void* const* key_pools, void* const* value_pools,
                                         const void* const* key_srcs, const void* const* value_srcs,
                                         int32_t layers, int64_t batch, int64_t heads, int64_t rows, int64_t dim,
                                         int64_t capacity, int64_t length, const int64_t* key_src_strides,
                                         const int64_t* value_src_strides, int32_t elem_bytes,
                                         const int64_t* chosen, int64_t chosen_stride_b, int64_t chosen_stride_w,
                                         int64_t past, int64_t extension, int64_t width, void* stream) {
  LaunchPlan* plan = nullptr;
  const int st = prepare_fold(key_pools, value_pools, key_srcs, value_srcs, layers, batch, heads, rows, dim,
                              capacity, length, key_src_strides, value_src_strides, elem_bytes, chosen,
                              chosen_stride_b, chosen_stride_w, past, extension, width, &plan);
  return launch_once(st, plan, stream);
}

extern "C" int speckv_append_commit_rows_prepare(void* const* key_pools, void* const* value_pools,
                                                 const void* const* key_srcs, const void* const* value_srcs,
                                                 int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                                                 int64_t dim, int64_t capacity, int64_t length,
                                                 const int64_t* key_src_strides, const int64_t* value_src_strides,
                                                 int32_t elem_bytes, const int64_t* chosen, int64_t chosen_stride_b,
                                                 int64_t chosen_stride_w, int64_t past, int64_t extension,
                                                 int64_t width, void** plan) {
  if (plan == nullptr) return fail(SPECKV_EINVAL, "speckv_append_commit_rows_prepare: null plan");
  LaunchPlan* p = nullptr;
  const int st = prepare_fold(key_pools, value_pools, key_srcs, value_srcs, layers, batch, heads, rows, dim,
                              capacity, length, key_src_strides, value_src_strides, elem_bytes, chosen,
                              chosen_stride_b, chosen_stride_w, past, extension, width, &p);
  *plan = st ? nullptr : p;
  return st;
}

extern "C" int speckv_plan_launch(const void* plan, void* stream) {
  if (plan == nullptr) return fail(SPECKV_EINVAL, "speckv_plan_launch: null plan");
  const LaunchPlan* p = static_cast<const LaunchPlan*>(plan);
  int dev = -1;
  if (p->device >= 0 && (cudaGetDevice(&dev) != cudaSuccess || dev != p->device))
    return fail(SPECKV_EINVAL, "speckv_plan_launch: plan prepared on cuda:%d, current device is cuda:%d", p->device,
                dev);
  return p->launch(static_cast<cudaStream_t>(stream));
}

extern "C" void speckv_plan_release(void* plan) { delete static_cast<LaunchPlan*>(plan); }

namespace speckv {
namespace {
int prepare_fold(void* const* key_pools, void* const* value_pools, const void* const* key_srcs,
                         const void* const* value_srcs, int32_t layers, int64_t batch, int64_t heads, int64_t rows,
                         int64_t dim, int64_t capacity, int64_t length, const int64_t* key_src_strides,
                         const int64_t* value_src_strides, int32_t elem_bytes, const int64_t* chosen,
                         int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past, int64_t extension,
                         int64_t width, LaunchPlan** out) {
  const char* fn = "speckv_append_commit_rows";
  if (extension < 0 || width < extension || past < 0 || past + width > capacity)
    return fail(SPECKV_EINVAL, "%s: extension %lld / width %lld / past %lld do not fit capacity %lld", fn,
                (long long)extension, (long long)width, (long long)past, (long long)capacity);
  if (width > extension && chosen == nullptr) return fail(SPECKV_EINVAL, "%s: null chosen", fn);
  LaunchPlan* ap = nullptr;
  int st = prepare_append(key_pools, value_pools, key_srcs, value_srcs, layers, batch, heads, rows, dim, capacity,
                          length, key_src_strides, value_src_strides, elem_bytes, nullptr, 0, &ap);
  if (st) return st;
  AppendPlan* app = dynamic_cast<AppendPlan*>(ap);
  if (app == nullptr) {  // nothing to append
    if (batch == 0 || width == extension) {
      *out = ap;
      return SPECKV_OK;
    }
    delete ap;
    return fail(SPECKV_ENOSUPPORT, "%s: no rows to append; use speckv_compact_suffix", fn);
  }
  const long long nvec = app->g.nvec.d;
  const long long maxa = (rows * nvec + kFoldThreads - 1) / kFoldThreads;
  if ((width - extension) * nvec > (long long)kFoldThreads * kFoldMaxC || maxa > 32) {
    delete ap;
    return fail(SPECKV_ENOSUPPORT, "%s: %lld accepted and %lld new rows of %lld vectors exceed the register "
                "stage; use speckv_compact_suffix then speckv_append_rows", fn, (long long)(width - extension),
                (long long)rows, nvec);
  }
  st = check_current_device(fn, {chosen});
  if (st) {
    delete ap;
    return st;
  }
  unsigned long long* err = device_error_word();
  if (err == nullptr) {
    delete ap;
    return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  }
  const long long groups = 2ll * layers * batch * heads;
  if (!fits_u31(groups)) {
    delete ap;
    return fail(SPECKV_ENOSUPPORT, "%s: too many groups", fn);
  }
  FoldPlan* plan = new FoldPlan();
  plan->device = app->device;
  plan->dst = app->dst;
  plan->src = app->src;
  plan->vec = app->vec;
  plan->g.a = app->g;
  plan->g.bh = FastDiv((uint32_t)(batch * heads));
  plan->g.chosen = chosen;
  plan->g.csb = chosen_stride_b;
  plan->g.csw = chosen_stride_w;
  plan->g.past = past;
  plan->g.capacity = capacity;
  plan->g.ext = (int)extension;
  plan->g.width = (int)width;
  plan->g.err = err;
  plan->maxa = maxa <= 8 ? 8 : (maxa <= 16 ? 16 : 32);
  plan->grid = (unsigned)groups;
  delete ap;
  *out = plan;
  return SPECKV_OK;
}

int prepare_append(void* const* key_pools, void* const* value_pools, const void* const* key_srcs,
                           const void* const* value_srcs, int32_t layers, int64_t batch, int64_t heads,
                           int64_t rows, int64_t dim, int64_t capacity, int64_t length,
                           const int64_t* key_src_strides, const int64_t* value_src_strides, int32_t elem_bytes,
                           const int64_t* row_table, int64_t pool_rows, LaunchPlan** out) {
  const char* fn = "speckv_append_rows";
  int st = check_common(fn, key_pools, value_pools, layers, heads, dim, capacity, elem_bytes);
  if (st) return st;
  st = check_table(fn, row_table, pool_rows, batch);
  if (st) return st;
  if (key_srcs == nullptr || value_srcs == nullptr || key_src_strides == nullptr || value_src_strides == nullptr)
    return fail(SPECKV_EINVAL, "%s: null source table or strides", fn);
  if (batch < 0 || rows < 0 || length < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (length + rows > capacity)
    return fail(SPECKV_EINVAL, "%s: length %lld + rows %lld exceeds capacity %lld", fn, (long long)length,
                (long long)rows, (long long)capacity);
  if (batch == 0 || rows == 0) {
    *out = new EmptyPlan();
    return SPECKV_OK;
  }
  const long long row_bytes = dim * elem_bytes;
  long long vals[4 * SPECKV_MAX_LAYERS + 8];
  int n = 0;
  vals[n++] = row_bytes;
  for (int k = 0; k < 3; ++k) {
    vals[n++] = key_src_strides[k] * elem_bytes;
    vals[n++] = value_src_strides[k] * elem_bytes;
  }
  SrcTable src;
  for (int l = 0; l < layers; ++l) {
    if (key_srcs[l] == nullptr || value_srcs[l] == nullptr)
      return fail(SPECKV_EINVAL, "%s: null source for layer %d", fn, l);
    src.ptr[2 * l] = static_cast<const char*>(key_srcs[l]);
    src.ptr[2 * l + 1] = static_cast<const char*>(value_srcs[l]);
    vals[n++] = (long long)(uintptr_t)key_srcs[l];
    vals[n++] = (long long)(uintptr_t)value_srcs[l];
    vals[n++] = (long long)(uintptr_t)key_pools[l];
    vals[n++] = (long long)(uintptr_t)value_pools[l];
  }
  const int vec = pick_vec(vals, n);
  const long long nvec = row_bytes / vec;
  const long long total = batch * heads * rows * nvec;
  if (!fits_u31(total)) return fail(SPECKV_ENOSUPPORT, "%s: %lld vectors per tensor exceeds 2^31", fn, total);
  st = check_current_device(fn, {key_pools[0], value_pools[0], key_srcs[0], value_srcs[0], row_table});
  if (st) return st;
  AppendPlan* plan = new AppendPlan();
  cudaGetDevice(&plan->device);
  PoolTable& dst = plan->dst;
  fill_pools(dst, key_pools, value_pools, layers);
  AppendGeom& g = plan->g;
  g.nvec = FastDiv((uint32_t)nvec);
  g.rows = FastDiv((uint32_t)rows);
  g.heads = FastDiv((uint32_t)heads);
  g.row_bytes = row_bytes;
  g.dst_sh = capacity * row_bytes;
  g.dst_sb = heads * g.dst_sh;
  g.dst_t0 = length * row_bytes;
  for (int kv = 0; kv < 2; ++kv) {
    const int64_t* s = kv ? value_src_strides : key_src_strides;
    g.src_sb[kv] = s[0] * elem_bytes;
    g.src_sh[kv] = s[1] * elem_bytes;
    g.src_st[kv] = s[2] * elem_bytes;
  }
  g.total = (uint32_t)total;
  g.rt = RowTable{row_table, pool_rows};
  g.err = nullptr;
  if (row_table != nullptr) {
    g.err = device_error_word();
    if (g.err == nullptr) {
      delete plan;
      return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
    }
  }
  constexpr int UNROLL = 4;
  plan->src = src;
  plan->vec = vec;
  plan->grid = dim3((unsigned)((total + kThreads * UNROLL - 1) / (kThreads * UNROLL)), 2 * layers);
  *out = plan;
  return SPECKV_OK;
}
}  // namespace
}  // namespace speckv

extern "C" int speckv_compact_suffix(void* const* key_pools, void* const* value_pools, int32_t layers,
                                     int64_t batch, int64_t heads, int64_t dim, int64_t capacity,
                                     int64_t length, const int64_t* chosen, int64_t chosen_stride_b,
                                     int64_t chosen_stride_w, int64_t past, int64_t extension,
                                     int64_t width, int32_t elem_bytes, const int64_t* row_table,
                                     int64_t pool_rows, void* stream) {
  const char* fn = "speckv_compact_suffix";
  int st = check_common(fn, key_pools, value_pools, layers, heads, dim, capacity, elem_bytes);
  if (st) return st;
  st = check_table(fn, row_table, pool_rows, batch);
  if (st) return st;
  if (batch < 0 || past < 0 || extension < 0 || width < 0 || length < 0)
    return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (extension > width) return fail(SPECKV_EINVAL, "%s: extension %lld > width %lld", fn, (long long)extension, (long long)width);
  if (past + width > length || length > capacity)
    return fail(SPECKV_EINVAL, "%s: past %lld + width %lld exceeds length %lld (capacity %lld)", fn,
                (long long)past, (long long)width, (long long)length, (long long)capacity);
  if (batch == 0 || extension == width) return SPECKV_OK;
  if (chosen == nullptr) return fail(SPECKV_EINVAL, "%s: null chosen", fn);
  st = check_current_device(fn, {key_pools[0], value_pools[0], chosen, row_table});
  if (st) return st;
  const long long row_bytes = dim * elem_bytes;
  const int vec = pool_vec(key_pools, value_pools, layers, row_bytes);
  const long long nvec = row_bytes / vec;
  const long long n = width - extension;
  const long long groups = 2ll * layers * batch * heads;
  if (!fits_u31(groups * 32) || !fits_u31(n * nvec))
    return fail(SPECKV_ENOSUPPORT, "%s: problem too large for 32-bit indexing", fn);
  PoolTable pools;
  fill_pools(pools, key_pools, value_pools, layers);
  CompactGeom g;
  g.bh = FastDiv((uint32_t)(batch * heads));
  g.heads = FastDiv((uint32_t)heads);
  g.nvec = FastDiv((uint32_t)nvec);
  g.row_bytes = row_bytes;
  g.sh = capacity * row_bytes;
  g.sb = heads * g.sh;
  g.length = length;
  g.past = past;
  g.extension = extension;
  g.csb = chosen_stride_b;
  g.csw = chosen_stride_w;
  g.n = (uint32_t)n;
  g.groups = (uint32_t)groups;
  g.rt = RowTable{row_table, pool_rows};
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  constexpr int MAXR = 8;
  if (n * nvec <= 32 * MAXR) {
    dim3 grid((unsigned)((groups * 32 + kThreads - 1) / kThreads));
    SPECKV_DISPATCH_VEC(vec, compact_warp_kernel<V, MAXR><<<grid, kThreads, 0, s>>>(pools, chosen, g, err));
  } else {
    const long long smem = n * row_bytes;
    if (smem > 200 * 1024) return fail(SPECKV_ENOSUPPORT, "%s: %lld rows of %lld bytes exceed the on-chip stage", fn, n, row_bytes);
    SPECKV_DISPATCH_VEC(vec, {
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(compact_smem_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      compact_smem_kernel<V><<<(unsigned)groups, kThreads, (size_t)smem, s>>>(pools, chosen, g, err);
    });
  }
  return check_launch(fn);
}

extern "C" int speckv_commit_round(void* const* key_pools, void* const* value_pools, int32_t layers,
                                   int64_t batch, int64_t heads, int64_t dim, int64_t capacity, int64_t length,
                                   int32_t elem_bytes, const int64_t* chosen, int64_t chosen_stride_b,
                                   int64_t chosen_stride_w, int64_t past, const int64_t* packet,
                                   int64_t packet_stride, int64_t max_width, uint8_t* pad_rows,
                                   int64_t pad_rows_stride, int64_t pad_rows_count, const int64_t* owners,
                                   uint8_t* pad_live, int64_t pad_live_stride, const uint8_t* newly_padded,
                                   int64_t np_stride_b, int64_t* positions, int64_t positions_stride_b,
                                   int64_t* past_positions, const int64_t* row_table, int64_t pool_rows,
                                   void* stream) {
  LaunchPlan* plan = nullptr;
  const int st = prepare_commit(key_pools, value_pools, layers, batch, heads, dim, capacity, length, elem_bytes,
                                chosen, chosen_stride_b, chosen_stride_w, past, packet, packet_stride, max_width,
                                pad_rows, pad_rows_stride, pad_rows_count, owners, pad_live, pad_live_stride,
                                newly_padded, np_stride_b, positions, positions_stride_b, past_positions, row_table,
                                pool_rows, &plan);
  return launch_once(st, plan, stream);
}

extern "C" int speckv_commit_round_prepare(void* const* key_pools, void* const* value_pools, int32_t layers,
                                           int64_t batch, int64_t heads, int64_t dim, int64_t capacity,
                                           int64_t length, int32_t elem_bytes, const int64_t* chosen,
                                           int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past,
                                           const int64_t* packet, int64_t packet_stride, int64_t max_width,
                                           uint8_t* pad_rows, int64_t pad_rows_stride, int64_t pad_rows_count,
                                           const int64_t* owners, uint8_t* pad_live, int64_t pad_live_stride,
                                           const uint8_t* newly_padded, int64_t np_stride_b, int64_t* positions,
                                           int64_t positions_stride_b, int64_t* past_positions,
                                           const int64_t* row_table, int64_t pool_rows, void** plan) {
  if (plan == nullptr) return fail(SPECKV_EINVAL, "speckv_commit_round_prepare: null plan");
  LaunchPlan* p = nullptr;
  const int st = prepare_commit(key_pools, value_pools, layers, batch, heads, dim, capacity, length, elem_bytes,
                                chosen, chosen_stride_b, chosen_stride_w, past, packet, packet_stride, max_width,
                                pad_rows, pad_rows_stride, pad_rows_count, owners, pad_live, pad_live_stride,
                                newly_padded, np_stride_b, positions, positions_stride_b, past_positions, row_table,
                                pool_rows, &p);
  *plan = st ? nullptr : p;
  return st;
}

namespace speckv {
namespace {
int prepare_commit(void* const* key_pools, void* const* value_pools, int32_t layers, int64_t batch,
                           int64_t heads, int64_t dim, int64_t capacity, int64_t length, int32_t elem_bytes,
                           const int64_t* chosen, int64_t chosen_stride_b, int64_t chosen_stride_w, int64_t past,
                           const int64_t* packet, int64_t packet_stride, int64_t max_width, uint8_t* pad_rows,
                           int64_t pad_rows_stride, int64_t pad_rows_count, const int64_t* owners,
                           uint8_t* pad_live, int64_t pad_live_stride, const uint8_t* newly_padded,
                           int64_t np_stride_b, int64_t* positions, int64_t positions_stride_b,
                           int64_t* past_positions, const int64_t* row_table, int64_t pool_rows,
                           LaunchPlan** out) {
  const char* fn = "speckv_commit_round";
  if (layers != 0) {
    int st = check_common(fn, key_pools, value_pools, layers, heads, dim, capacity, elem_bytes);
    if (st) return st;
    st = check_table(fn, row_table, pool_rows, batch);
    if (st) return st;
  }
  if (batch < 0 || past < 0 || max_width < 1 || length < 0) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (layers != 0 && (past > length || length > capacity))
    return fail(SPECKV_EINVAL, "%s: past %lld / length %lld / capacity %lld inconsistent", fn, (long long)past,
                (long long)length, (long long)capacity);
  if (batch == 0 || (layers == 0 && positions == nullptr)) {
    *out = new EmptyPlan();
    return SPECKV_OK;
  }
  if (packet == nullptr || packet_stride < 3) return fail(SPECKV_EINVAL, "%s: packet rows need 3 columns", fn);
  if (layers != 0 && chosen == nullptr) return fail(SPECKV_EINVAL, "%s: null chosen", fn);
  if (positions != nullptr) {
    if (!newly_padded || !past_positions) return fail(SPECKV_EINVAL, "%s: null position operand", fn);
    if (pad_rows != nullptr && (owners == nullptr || past + max_width > pad_rows_stride))
      return fail(SPECKV_EINVAL, "%s: padding rows need owners and past + width <= row stride", fn);
    if (pad_live != nullptr && past + max_width > pad_live_stride)
      return fail(SPECKV_EINVAL, "%s: past + width exceeds live padding row stride", fn);
  }
  constexpr int MAXR = 16;
  const long long row_bytes = layers != 0 ? dim * elem_bytes : 16;
  const int vec = layers != 0 ? pool_vec(key_pools, value_pools, layers, row_bytes) : 16;
  const long long nvec = row_bytes / vec;
  if (!fits_u31(length)) return fail(SPECKV_ENOSUPPORT, "%s: length exceeds 2^31", fn);
  if (layers != 0 && max_width * nvec > 32 * MAXR)
    return fail(SPECKV_ENOSUPPORT, "%s: %lld rows of %lld vectors exceed the register stage", fn,
                (long long)max_width, nvec);
  const long long groups = 2ll * layers * batch * (layers != 0 ? heads : 0);
  const long long compact_blocks = (groups + kThreads / 32 - 1) / (kThreads / 32);
  const long long position_blocks = positions != nullptr ? (batch + kThreads / 32 - 1) / (kThreads / 32) : 0;
  if (!fits_u31(groups) || !fits_u31(compact_blocks + position_blocks) || !fits_u31(batch * (layers != 0 ? heads : 1)))
    return fail(SPECKV_ENOSUPPORT, "%s: problem too large for 32-bit indexing", fn);
  const void* k0 = layers != 0 ? key_pools[0] : nullptr;
  const void* v0 = layers != 0 ? value_pools[0] : nullptr;
  const int dst = check_current_device(fn, {k0, v0, packet, chosen, row_table, pad_rows, owners, pad_live,
                                            newly_padded, positions, past_positions});
  if (dst) return dst;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  CommitPlan* plan = new CommitPlan();
  cudaGetDevice(&plan->device);
  PoolTable& pools = plan->pools;
  if (layers != 0) fill_pools(pools, key_pools, value_pools, layers);
  RoundGeom& g = plan->g;
  g.c.bh = FastDiv((uint32_t)(batch * (layers != 0 ? heads : 1)));
  g.c.heads = FastDiv((uint32_t)(layers != 0 ? heads : 1));
  g.c.nvec = FastDiv((uint32_t)nvec);
  g.c.row_bytes = row_bytes;
  g.c.sh = layers != 0 ? capacity * row_bytes : 0;
  g.c.sb = layers != 0 ? heads * g.c.sh : 0;
  g.c.length = layers != 0 ? length : past + max_width;
  g.c.past = past;
  g.c.extension = 0;
  g.c.csb = chosen_stride_b;
  g.c.csw = chosen_stride_w;
  g.c.n = 0;
  g.c.groups = (uint32_t)groups;
  g.c.rt = RowTable{layers != 0 ? row_table : nullptr, pool_rows};
  g.chosen = chosen;
  g.packet = packet;
  g.ps = packet_stride;
  g.batch = (uint32_t)batch;
  g.max_width = (uint32_t)max_width;
  g.compact_blocks = (uint32_t)compact_blocks;
  g.pos = PositionArgs{pad_rows, pad_rows_stride, pad_rows_count, owners, pad_live, pad_live_stride,
                       newly_padded, np_stride_b, positions, positions_stride_b, past_positions};
  plan->err = err;
  plan->vec = vec;
  plan->grid = (unsigned)(compact_blocks + position_blocks);
  // register stage sized to the widest round the schedule allows (fewer registers, more resident warps)
  const long long stage = max_width * nvec;
  plan->maxr = stage <= 32 * 4 ? 4 : (stage <= 32 * 8 ? 8 : MAXR);
  *out = plan;
  return SPECKV_OK;
}
}  // namespace
}  // namespace speckv

// A CTA stages every batch row of up to kStageBytes / (rows * row bytes)
// positions; a single position of all rows may take up to 3 * kStageBytes.
static const long long kStageBytes = 64 * 1024;

extern "C" int64_t speckv_remap_scratch_bytes(int64_t new_batch, int64_t heads, int64_t dim, int64_t length,
                                              int32_t elem_bytes) {
  if (new_batch <= 0 || heads <= 0 || dim <= 0 || length <= 0 || elem_bytes <= 0) return 0;
  if (new_batch * dim * elem_bytes <= 3 * kStageBytes) return 0;
  return 2 * new_batch * heads * length * dim * elem_bytes;
}

extern "C" int speckv_remap_rows(void* const* key_pools, void* const* value_pools, int32_t layers,
                                 const int64_t* indices, int64_t new_batch, int64_t batch_capacity,
                                 int64_t heads, int64_t dim, int64_t capacity, int64_t length,
                                 void* scratch, int64_t scratch_bytes, int32_t elem_bytes, void* stream) {
  const char* fn = "speckv_remap_rows";
  int st = check_common(fn, key_pools, value_pools, layers, heads, dim, capacity, elem_bytes);
  if (st) return st;
  if (new_batch < 0 || length < 0 || batch_capacity < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (new_batch > batch_capacity)
    return fail(SPECKV_EINVAL, "%s: new batch %lld exceeds batch capacity %lld", fn, (long long)new_batch,
                (long long)batch_capacity);
  if (length > capacity) return fail(SPECKV_EINVAL, "%s: length exceeds capacity", fn);
  if (new_batch == 0 || length == 0) return SPECKV_OK;
  if (indices == nullptr) return fail(SPECKV_EINVAL, "%s: null indices", fn);
  st = check_current_device(fn, {key_pools[0], value_pools[0], indices, scratch});
  if (st) return st;
  if (!fits_u31(batch_capacity) || !fits_u31(length)) return fail(SPECKV_ENOSUPPORT, "%s: sizes exceed 2^31", fn);
  const long long row_bytes = dim * elem_bytes;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long per_position = new_batch * row_bytes;  // stage bytes for one position
  if (speckv_remap_scratch_bytes(new_batch, heads, dim, length, elem_bytes) == 0) {
    const int vec = pool_vec(key_pools, value_pools, layers, row_bytes);
    const long long nvec = row_bytes / vec;
    long long tile = per_position <= kStageBytes ? kStageBytes / per_position : 1;
    if (tile > length) tile = length;
    const long long tiles = (length + tile - 1) / tile;
    const long long smem = new_batch * tile * row_bytes;
    if (!fits_u31(heads * tiles) || !fits_u31(new_batch * tile * nvec))
      return fail(SPECKV_ENOSUPPORT, "%s: problem too large for 32-bit indexing", fn);
    PoolTable pools;
    fill_pools(pools, key_pools, value_pools, layers);
    RemapGeom g;
    g.row_vecs = FastDiv((uint32_t)(tile * nvec));
    g.nvec = FastDiv((uint32_t)nvec);
    g.tiles = FastDiv((uint32_t)tiles);
    g.row_bytes = row_bytes;
    g.sh = capacity * row_bytes;
    g.sb = heads * g.sh;
    g.new_batch = (uint32_t)new_batch;
    g.batch_cap = (uint32_t)batch_capacity;
    g.tile = (uint32_t)tile;
    g.length = (uint32_t)length;
    dim3 grid((unsigned)(heads * tiles), 2 * layers);
    SPECKV_DISPATCH_VEC(vec, {
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(remap_smem_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      remap_smem_kernel<V><<<grid, kThreads, (size_t)smem, s>>>(pools, indices, g, err);
    });
    return check_launch(fn);
  }
  // Two-phase path through caller scratch, one layer at a time.
  const long long need = 2 * new_batch * heads * length * row_bytes;
  if (scratch == nullptr || scratch_bytes < need)
    return fail(SPECKV_EINVAL, "%s: %lld rows per position need %lld scratch bytes, got %lld", fn,
                (long long)new_batch, need, (long long)scratch_bytes);
  long long vals[2 * SPECKV_MAX_LAYERS + 2];
  int nv = 0;
  vals[nv++] = row_bytes;
  vals[nv++] = (long long)(uintptr_t)scratch;
  for (int l = 0; l < layers; ++l) {
    vals[nv++] = (long long)(uintptr_t)key_pools[l];
    vals[nv++] = (long long)(uintptr_t)value_pools[l];
  }
  const int vec = pick_vec(vals, nv);
  RemapScratchGeom g;
  g.row_bytes = row_bytes;
  g.nvec = row_bytes / vec;
  g.length = length;
  g.heads = heads;
  g.sh = capacity * row_bytes;
  g.sb = heads * g.sh;
  g.new_batch = new_batch;
  g.batch_cap = batch_capacity;
  g.per_tensor = new_batch * heads * length * g.nvec;
  long long blocks = (g.per_tensor + kThreads - 1) / kThreads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  dim3 grid((unsigned)blocks, 2);
  char* scr = static_cast<char*>(scratch);
  for (int l = 0; l < layers; ++l) {
    char* kp = static_cast<char*>(key_pools[l]);
    char* vp = static_cast<char*>(value_pools[l]);
    SPECKV_DISPATCH_VEC(vec, {
      remap_gather_kernel<V><<<grid, kThreads, 0, s>>>(kp, vp, indices, scr, g, err);
      remap_scatter_kernel<V><<<grid, kThreads, 0, s>>>(kp, vp, indices, scr, g);
    });
    st = check_launch(fn);
    if (st) return st;
  }
  return SPECKV_OK;
}

extern "C" int speckv_move_rows(void* const* key_pools, void* const* value_pools, int32_t layers,
                                const int64_t* sources, const int64_t* destinations, int64_t count,
                                int64_t batch_capacity, int64_t heads, int64_t dim, int64_t capacity,
                                int64_t length, int32_t elem_bytes, void* stream) {
  const char* fn = "speckv_move_rows";
  int st = check_common(fn, key_pools, value_pools, layers, heads, dim, capacity, elem_bytes);
  if (st) return st;
  if (count < 0 || length < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (length > capacity) return fail(SPECKV_EINVAL, "%s: length exceeds capacity", fn);
  if (count == 0 || length == 0) return SPECKV_OK;
  if (sources == nullptr || destinations == nullptr) return fail(SPECKV_EINVAL, "%s: null index list", fn);
  st = check_current_device(fn, {key_pools[0], value_pools[0], sources, destinations});
  if (st) return st;
  if (!fits_u31(batch_capacity)) return fail(SPECKV_ENOSUPPORT, "%s: batch capacity exceeds 2^31", fn);
  const long long row_bytes = dim * elem_bytes;
  const int vec = pool_vec(key_pools, value_pools, layers, row_bytes);
  const long long nvec = row_bytes / vec;
  const long long span = length * nvec;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  PoolTable pools;
  fill_pools(pools, key_pools, value_pools, layers);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  constexpr int UNROLL = 4;
  // Chunk the row list so each launch stays within 32-bit indexing.
  long long per_row = heads * span;
  if (!fits_u31(per_row)) return fail(SPECKV_ENOSUPPORT, "%s: one row exceeds 2^31 vectors", fn);
  long long rows_per_launch = ((1ll << 31) - 1) / per_row;
  for (long long j0 = 0; j0 < count; j0 += rows_per_launch) {
    const long long c = (count - j0) < rows_per_launch ? (count - j0) : rows_per_launch;
    MoveGeom g;
    g.span = FastDiv((uint32_t)span);
    g.heads = FastDiv((uint32_t)heads);
    g.sh = capacity * row_bytes;
    g.sb = heads * g.sh;
    g.batch_cap = (uint32_t)batch_capacity;
    g.total = (uint32_t)(c * per_row);
    dim3 grid((unsigned)((g.total + kThreads * UNROLL - 1) / (kThreads * UNROLL)), 2 * layers);
    SPECKV_DISPATCH_VEC(vec, move_rows_kernel<V, UNROLL><<<grid, kThreads, 0, s>>>(pools, sources + j0, destinations + j0, g, err));
    st = check_launch(fn);
    if (st) return st;
  }
  return SPECKV_OK;
}
