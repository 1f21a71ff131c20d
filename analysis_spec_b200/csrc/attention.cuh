// Argument block shared by the tree-verify attention paths.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace speckv {

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* mask;         // dense additive (batch, 1, rows, kv_len) contiguous, or null
  const uint32_t* bits;     // or bit-packed visibility (batch, rows, row_words)
  long long row_words;
  const int* first_col;     // optional with bits: first visible column per sequence
  void* out;                // (batch, rows, q_heads, dim) contiguous
  long long qs[3], ks[3], vs[3];  // element strides (b, h, t); dim stride is 1
  long long batch, q_heads, kv_heads, rows, kv_len, dim;
  float scale;
  int dtype, mask_dtype;
  const int64_t* row_table;  // optional (bits path): pool row of each sequence's K/V
  long long kv_batch;        // rows of the K/V tensors (>= batch without a table)
  // Fused append (bits path, past >= 0): k / v are the pools holding `past` cached positions
  // with room for `rows` more (kv_len = past + rows); k_new / v_new, (batch, kv_heads, rows,
  // dim) strided views, are attended as the last keys and stored into the pools at past.
  long long past;            // < 0: no append
  const void* k_new;
  const void* v_new;
  long long kns[3], vns[3];
};

// CUDA-core path (any head dim <= 256, any dtype).
int attention_generic(const AttnArgs& a, cudaStream_t s);

// tcgen05 / TMEM / TMA path: head dim 128, bf16 or fp16, 16-byte aligned rows.
bool sm100_supported(const AttnArgs& a);
int attention_sm100(const AttnArgs& a, cudaStream_t s);

// Test hooks of the tensor-core kernels on the current device (synchronous copies):
// the bounded waits' limit in ns (<= 0: the default 2 s) and whether CTA 0 of the
// visibility-bits kernel withholds its first Q-tile arrival.
int attention_test_hooks(long long wait_limit_ns, int withhold_q_arrival);

// Upper bound on the persistent attention grid for this process (<= 0: one CTA per SM).
void attention_set_ctas(int ctas);

// Key-range chunks of long sequences in the visibility-bits kernel (0: off, the default).
void attention_set_chunks(int on);

// Zeroes the merge counters of split attention items (all slots): a launch leaves them at zero
// when it completes; after a launch that ended in an error they may not be.
int attention_reset_partials();

}  // namespace speckv
