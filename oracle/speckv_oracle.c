/*
 * CPU restatement of the reference's KV row movement, used ONLY as test
 * infrastructure: the parity checker of the CUDA kernels and the timed CPU
 * baseline. The product never links or calls this file.
 *
 * Byte-generic: every pool is (batch_capacity, heads, capacity, dim) contiguous
 * with rows of dim * es bytes. OpenMP spreads (sequence, head) slabs over the
 * host cores.
 *
 * Followed reference code (nhatminz/analysis_spec):
 *   oracle_append          helper/opd_static_cache.py:104-108 (StaticAppendLayer.update)
 *   oracle_compact_suffix  helper/opd_scheduling.py:357-380 (compact_suffix_inplace)
 *   oracle_remap_rows      helper/opd_kv_kernels.py:11-40 (gather to scratch, then scatter)
 *                          and its CPU branch helper/opd_static_cache.py:134-142
 *   oracle_move_rows       helper/opd_kv_kernels.py:43-58 and helper/opd_static_cache.py:165-168
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static inline uint8_t* row_ptr(uint8_t* pool, int64_t b, int64_t h, int64_t t, int64_t heads, int64_t cap,
                               int64_t row) {
  return pool + ((b * heads + h) * cap + t) * row;
}

/* pool[b][h][length + t] = src[b][h][t]; src element strides s[0..2] (b, h, t), unit on dim. */
void oracle_append(uint8_t* kpool, uint8_t* vpool, const uint8_t* ksrc, const uint8_t* vsrc, int64_t batch,
                   int64_t heads, int64_t rows, int64_t dim, int64_t cap, int64_t length, const int64_t* ks,
                   const int64_t* vs, int32_t es) {
  const int64_t row = dim * es;
  for (int kv = 0; kv < 2; ++kv) {
    uint8_t* pool = kv ? vpool : kpool;
    const uint8_t* src = kv ? vsrc : ksrc;
    const int64_t* s = kv ? vs : ks;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b)
      for (int64_t h = 0; h < heads; ++h)
        for (int64_t t = 0; t < rows; ++t)
          memcpy(row_ptr(pool, b, h, length + t, heads, cap, row), src + (b * s[0] + h * s[1] + t * s[2]) * es,
                 (size_t)row);
  }
}

/* Gathers rows chosen[b][extension..width) of every (b, h) into a scratch, then
 * writes them to [past + extension, past + width). Returns the number of
 * out-of-range chosen entries (those rows are skipped). */
int64_t oracle_compact_suffix(uint8_t* key, uint8_t* value, int64_t batch, int64_t heads, int64_t dim, int64_t cap,
                              int64_t length, const int64_t* chosen, int64_t csb, int64_t csw, int64_t past,
                              int64_t extension, int64_t width, int32_t es) {
  const int64_t n = width - extension;
  if (n <= 0 || batch <= 0) return 0;
  const int64_t row = dim * es;
  uint8_t* scratch = (uint8_t*)malloc((size_t)(batch * heads * n * row));
  int64_t bad = 0;
  for (int kv = 0; kv < 2; ++kv) {
    uint8_t* pool = kv ? value : key;
#pragma omp parallel for collapse(2) schedule(static) reduction(+ : bad)
    for (int64_t b = 0; b < batch; ++b)
      for (int64_t h = 0; h < heads; ++h)
        for (int64_t j = 0; j < n; ++j) {
          const int64_t pos = chosen[b * csb + (extension + j) * csw];
          if (pos < 0 || pos >= length) {
            bad += 1;
            continue;
          }
          memcpy(scratch + ((b * heads + h) * n + j) * row, row_ptr(pool, b, h, pos, heads, cap, row), (size_t)row);
        }
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b)
      for (int64_t h = 0; h < heads; ++h)
        for (int64_t j = 0; j < n; ++j) {
          const int64_t pos = chosen[b * csb + (extension + j) * csw];
          if (pos < 0 || pos >= length) continue;
          memcpy(row_ptr(pool, b, h, past + extension + j, heads, cap, row),
                 scratch + ((b * heads + h) * n + j) * row, (size_t)row);
        }
  }
  free(scratch);
  return bad;
}

/* pool[i] = pool[indices[i]] over positions [0, length), i < new_batch, via a
 * scratch holding every gathered row first. Returns the count of indices
 * outside [0, batch_capacity) (skipped). */
int64_t oracle_remap_rows(uint8_t* kpool, uint8_t* vpool, const int64_t* indices, int64_t new_batch,
                          int64_t batch_capacity, int64_t heads, int64_t dim, int64_t cap, int64_t length,
                          int32_t es) {
  if (new_batch <= 0 || length <= 0) return 0;
  const int64_t row = dim * es;
  const int64_t slab = length * row;  /* live bytes of one (sequence, head) */
  uint8_t* scratch = (uint8_t*)malloc((size_t)(new_batch * heads * slab));
  int64_t bad = 0;
  for (int64_t i = 0; i < new_batch; ++i)
    if (indices[i] < 0 || indices[i] >= batch_capacity) bad += 1;
  for (int kv = 0; kv < 2; ++kv) {
    uint8_t* pool = kv ? vpool : kpool;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t i = 0; i < new_batch; ++i)
      for (int64_t h = 0; h < heads; ++h) {
        const int64_t s = indices[i];
        if (s < 0 || s >= batch_capacity) continue;
        memcpy(scratch + (i * heads + h) * slab, row_ptr(pool, s, h, 0, heads, cap, row), (size_t)slab);
      }
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t i = 0; i < new_batch; ++i)
      for (int64_t h = 0; h < heads; ++h) {
        const int64_t s = indices[i];
        if (s < 0 || s >= batch_capacity) continue;
        memcpy(row_ptr(pool, i, h, 0, heads, cap, row), scratch + (i * heads + h) * slab, (size_t)slab);
      }
  }
  free(scratch);
  return bad;
}

/* pool[destinations[j]] = pool[sources[j]] over [0, length) (disjoint lists). */
int64_t oracle_move_rows(uint8_t* kpool, uint8_t* vpool, const int64_t* sources, const int64_t* destinations,
                         int64_t count, int64_t batch_capacity, int64_t heads, int64_t dim, int64_t cap,
                         int64_t length, int32_t es) {
  if (count <= 0 || length <= 0) return 0;
  const int64_t row = dim * es;
  const int64_t slab = length * row;
  int64_t bad = 0;
  for (int64_t j = 0; j < count; ++j)
    if (sources[j] < 0 || sources[j] >= batch_capacity || destinations[j] < 0 || destinations[j] >= batch_capacity)
      bad += 1;
  for (int kv = 0; kv < 2; ++kv) {
    uint8_t* pool = kv ? vpool : kpool;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t j = 0; j < count; ++j)
      for (int64_t h = 0; h < heads; ++h) {
        const int64_t s = sources[j], d = destinations[j];
        if (s < 0 || s >= batch_capacity || d < 0 || d >= batch_capacity) continue;
        memcpy(row_ptr(pool, d, h, 0, heads, cap, row), row_ptr(pool, s, h, 0, heads, cap, row), (size_t)slab);
      }
  }
  return bad;
}
