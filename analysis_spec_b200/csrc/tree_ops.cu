// Tree kernels of the verify round: greedy acceptance walk, gap-first padded
// commit layout (+ the one host packet), additive ancestor mask and the
// position / padding update after a commit. All integer work, exact.
//
// Semantics follow helper/tree_kernels.py:7-41, 68-155 and
// helper/tree_verification.py:19-42, 237-322 of the reference.
#include "common.cuh"
#include "positions.cuh"

#include <limits.h>

namespace speckv {
namespace {

// ---------------------------------------------------------------------------
// trace_path: one warp per sequence.
// ---------------------------------------------------------------------------
__global__ void trace_path_kernel(const int64_t* __restrict__ parents, const int64_t* __restrict__ tokens,
                                  const int64_t* __restrict__ contexts, const int64_t* __restrict__ samples,
                                  int64_t batch, int64_t rows, int64_t eos, int64_t* out_t, int64_t* out_i,
                                  int64_t* out_c, int64_t osb, int64_t osw, int64_t width, int64_t* lengths) {
  const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (b >= batch) return;
  const int64_t* P = parents + b * rows;
  const int64_t* T = tokens + b * rows;
  const int64_t* C = contexts + b * rows;
  const int64_t* S = samples + b * rows;
  int64_t cur = 0, length = 0;
  bool live = true;
  for (int64_t j = 0; j < width; ++j) {
    const int64_t tok = S[cur];
    if (lane == 0) {
      out_t[b * osb + j * osw] = live ? tok : -1;
      out_i[b * osb + j * osw] = live ? cur : -1;
      out_c[b * osb + j * osw] = live ? C[cur] : -1;
    }
    length += live ? 1 : 0;
    int64_t found = rows;
    if (live && tok != eos) {
      // first (lowest-index) non-root child of `cur` carrying the sampled token
      for (int64_t r0 = 0; r0 < rows; r0 += 32) {
        const int64_t r = r0 + lane;
        const bool m = r > 0 && r < rows && P[r] == cur && T[r] == tok;
        const unsigned bal = __ballot_sync(0xffffffffu, m);
        if (bal) {
          found = r0 + __ffs(bal) - 1;
          break;
        }
      }
    }
    live = live && found < rows && tok != eos;
    cur = found < rows - 1 ? found : rows - 1;
  }
  if (lane == 0) lengths[b] = length;
}

// ---------------------------------------------------------------------------
// pack_tree: one CTA per sequence; full -> packed row map in shared memory.
// ---------------------------------------------------------------------------
constexpr int kPackThreads = 128;

__global__ void __launch_bounds__(kPackThreads) pack_tree_kernel(const int64_t* __restrict__ full_parents,
                                                                 const int64_t* __restrict__ full_contexts,
                                                                 const int64_t* __restrict__ all_tokens,
                                                                 const int64_t* __restrict__ chosen, long long n,
                                                                 long long p, int64_t* out_parents, int64_t* out_tokens,
                                                                 int64_t* out_contexts, long long osb,
                                                                 unsigned long long* err) {
  extern __shared__ int inverse[];  // [n + 1]: full node + 1 -> packed row, -1 if not packed
  const long long b = blockIdx.x;
  const int64_t* fp = full_parents + b * n;
  const int64_t* ch = chosen + b * p;
  for (long long i = threadIdx.x; i <= n; i += kPackThreads) inverse[i] = i == 0 ? 0 : -1;
  __syncthreads();
  for (long long j = threadIdx.x; j < p; j += kPackThreads) {
    const long long c = ch[j];
    if (c >= 0 && c < n) inverse[c + 1] = (int)(j + 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    out_parents[b * osb] = -1;
    out_tokens[b * osb] = -1;
    out_contexts[b * osb] = 0;
  }
  for (long long j = threadIdx.x; j < p; j += kPackThreads) {
    const long long c = ch[j];
    long long parent = -1, tok = -1, ctx = -1;
    if (c >= 0 && c < n) {
      const long long fpar = fp[c];
      parent = (fpar >= -1 && fpar < n) ? inverse[fpar + 1] : -1;
      tok = all_tokens[b * n + c];
      ctx = full_contexts[b * n + c];
    }
    if (parent < 0 || parent > j) record_error(err, SPECKV_DERR_TREE_INDEX, j + 1);
    out_parents[b * osb + j + 1] = parent;
    out_tokens[b * osb + j + 1] = tok;
    out_contexts[b * osb + j + 1] = ctx;
  }
}

// ---------------------------------------------------------------------------
// padded layout / schedule: one CTA per sequence.
// ---------------------------------------------------------------------------
constexpr int kPadThreads = 128;

__device__ __forceinline__ long long block_reduce(long long v, bool is_max, long long* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? (w > v ? w : v) : (w < v ? w : v);
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int i = 1; i < kPadThreads / 32; ++i) v = is_max ? (red[i] > v ? red[i] : v) : (red[i] < v ? red[i] : v);
  return v;
}

struct PadArgs {
  const int64_t* tokens;
  long long tsb, tsw;
  const int64_t* indices;
  long long isb, isw;
  const int64_t* lengths;
  long long batch, capacity, width, past, eos;
  int64_t* ot;
  int64_t* oi;
  uint8_t* om;
  long long osb, osw;
  int64_t* last;
  long long last_stride;
  int64_t* packet;  // null for pad_verified_path
  long long psb, psw;
  const int64_t* snapshot;
};

__global__ void __launch_bounds__(kPadThreads) pad_kernel(PadArgs a) {
  extern __shared__ int src_of[];  // first accepted slot landing on each output position
  __shared__ long long red[kPadThreads / 32];
  const long long b = blockIdx.x;
  long long width = a.width;
  if (a.packet != nullptr) {  // schedule: width = max(lengths) over the whole batch
    long long w = LLONG_MIN;
    for (long long i = threadIdx.x; i < a.batch; i += kPadThreads) w = a.lengths[i] > w ? a.lengths[i] : w;
    width = block_reduce(w, true, red);
    if (width < 0) width = 0;
    if (width > a.capacity) width = a.capacity;
  }
  const long long length = a.lengths[b];
  long long budget = width - length;
  if (budget < 0) budget = 0;
  for (long long p = threadIdx.x; p < width; p += kPadThreads) src_of[p] = INT_MAX;
  __syncthreads();
  long long last = -1;
  for (long long s = threadIdx.x; s < a.capacity; s += kPadThreads) {
    if (s >= length) continue;
    const long long idx = a.indices[b * a.isb + s * a.isw];
    long long gap = idx - s;
    if (gap < 0) gap = 0;
    const long long dest = s + (gap < budget ? gap : budget);
    last = dest > last ? dest : last;
    if (dest >= 0 && dest < width) atomicMin(&src_of[dest], (int)s);
  }
  last = block_reduce(last, true, red);  // also orders the atomics before the reads below
  long long ext = width;
  for (long long p = threadIdx.x; p < width; p += kPadThreads) {
    const int s = src_of[p];
    const bool acc = s != INT_MAX;
    const long long tok = acc ? a.tokens[b * a.tsb + s * a.tsw] : a.eos;
    const long long ch = acc ? a.indices[b * a.isb + s * a.isw] : 0;
    const long long oid = acc ? ch + a.past : p + a.past;
    a.ot[b * a.osb + p * a.osw] = acc ? tok : a.eos;
    a.oi[b * a.osb + p * a.osw] = oid;
    a.om[b * a.osb + p * a.osw] = acc ? 0 : 1;
    if (oid != p + a.past && p < ext) ext = p;
    if (a.packet != nullptr) a.packet[b * a.psb + (3 + p) * a.psw] = acc ? -1 : oid;
  }
  if (threadIdx.x == 0) a.last[b * a.last_stride] = last;
  if (a.packet == nullptr) return;
  ext = block_reduce(ext, false, red);
  for (long long p = width + threadIdx.x; p < a.capacity; p += kPadThreads) a.packet[b * a.psb + (3 + p) * a.psw] = -1;
  if (threadIdx.x == 0) {
    a.packet[b * a.psb] = length;
    const long long tail = length > 0 ? a.tokens[b * a.tsb + (length - 1) * a.tsw] : a.eos + 1;
    a.packet[b * a.psb + a.psw] = tail == a.eos ? 1 : 0;
    a.packet[b * a.psb + 2 * a.psw] = ext;
    if (a.snapshot != nullptr) a.packet[b * a.psb + (a.capacity + 3) * a.psw] = *a.snapshot;
  }
}

// ---------------------------------------------------------------------------
// tree mask: CTA per (row, sequence, 1024-column chunk).
// ---------------------------------------------------------------------------
constexpr int kMaskThreads = 256;
constexpr int kMaskCols = 1024;
constexpr int kMaxSteps = 256;

// Masked entries hold the dtype's lowest finite value: -FLT_MAX (0xff7fffff),
// bf16 0xff7f, fp16 -65504 (0xfbff), matching torch.finfo(dtype).min.
__global__ void __launch_bounds__(kMaskThreads) tree_mask_kernel(const int64_t* __restrict__ parents, long long rows,
                                                                 long long past, long long steps, void* mask, int dtype,
                                                                 const uint8_t* __restrict__ pad, long long pad_sb,
                                                                 unsigned long long* err) {
  __shared__ long long anc[kMaxSteps];
  __shared__ int nanc;
  const long long r = blockIdx.x;
  const long long b = blockIdx.y;
  if (threadIdx.x == 0) {
    long long cur = r;
    int n = 0;
    for (long long k = 0; k < steps && k < kMaxSteps; ++k) {
      if (cur >= 0) anc[n++] = cur;
      const long long at = cur > 0 ? cur : 0;
      if (at >= rows) {
        record_error(err, SPECKV_DERR_TREE_INDEX, at);
        break;
      }
      cur = parents[b * rows + at];
    }
    nanc = n;
  }
  __syncthreads();
  const long long cols = past + rows;
  const long long row_off = (b * rows + r) * cols;
  const long long c0 = (long long)blockIdx.z * kMaskCols;
  for (long long c = c0 + threadIdx.x; c < c0 + kMaskCols && c < cols; c += kMaskThreads) {
    bool vis = c <= past;
    for (int k = 0; k < nanc && !vis; ++k) vis = c == past + anc[k];
    if (pad != nullptr && pad[b * pad_sb + c]) vis = false;
    if (dtype == SPECKV_F32) {
      static_cast<uint32_t*>(mask)[row_off + c] = vis ? 0u : 0xff7fffffu;
    } else if (dtype == SPECKV_BF16) {
      static_cast<uint16_t*>(mask)[row_off + c] = vis ? (uint16_t)0 : (uint16_t)0xff7f;
    } else {
      static_cast<uint16_t*>(mask)[row_off + c] = vis ? (uint16_t)0 : (uint16_t)0xfbff;
    }
  }
}

// ---------------------------------------------------------------------------
// bit-packed visibility: CTA per (row, sequence); thread per 32-column word.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kMaskThreads) tree_bits_kernel(const int64_t* __restrict__ parents, long long rows,
                                                                 long long past, long long steps,
                                                                 const uint8_t* __restrict__ pad, long long pad_sb,
                                                                 uint32_t* bits, long long row_words, int* first_col,
                                                                 unsigned long long* err) {
  __shared__ long long anc[kMaxSteps];
  __shared__ int nanc;
  const long long r = blockIdx.x;
  const long long b = blockIdx.y;
  if (threadIdx.x == 0) {
    long long cur = r;
    int n = 0;
    for (long long k = 0; k < steps && k < kMaxSteps; ++k) {
      if (cur >= 0) anc[n++] = cur;
      const long long at = cur > 0 ? cur : 0;
      if (at >= rows) {
        record_error(err, SPECKV_DERR_TREE_INDEX, at);
        break;
      }
      cur = parents[b * rows + at];
    }
    nanc = n;
  }
  __syncthreads();
  const long long cols = past + rows;
  uint32_t* out = bits + (b * rows + r) * row_words;
  for (long long w = threadIdx.x; w < row_words; w += kMaskThreads) {
    uint32_t word = 0;
    const long long c0 = w * 32;
    if (c0 < cols) {
      for (int i = 0; i < 32; ++i) {
        const long long c = c0 + i;
        if (c >= cols) break;
        bool vis = c <= past;
        for (int k = 0; k < nanc && !vis; ++k) vis = c == past + anc[k];
        if (vis && pad != nullptr && pad[b * pad_sb + c]) vis = false;
        word |= (vis ? 1u : 0u) << i;
      }
    }
    out[w] = word;
    if (r == 0 && word != 0) atomicMin(first_col + b, (int)(c0 + __ffs(word) - 1));
  }
}

// ---------------------------------------------------------------------------
// bit-packed visibility, CTA per sequence: the prefix words (columns 0 .. past,
// padding removed) are built once and shared by every row; each row adds its
// ancestors as a bitstring over the tree columns past .. past + rows - 1. Same
// words as tree_bits_kernel; no atomics (first_col is row 0's first visible column).
// ---------------------------------------------------------------------------
constexpr int kSeqBitsThreads = 256;
constexpr long long kSeqBitsMaxRows = 256;  // rows x ceil(rows / 32) ancestor words in shared memory

// bits [off, off + 32) of a bitstring of n words (bits outside it read as 0)
__device__ __forceinline__ uint32_t bit_window(const uint32_t* a, int n, long long off) {
  if (off <= -32 || off >= 32ll * n) return 0u;
  const long long q = off >= 0 ? off / 32 : -((31 - off) / 32);
  const int sh = (int)(off - 32 * q);
  const uint32_t lo = (q >= 0 && q < n) ? a[q] : 0u;
  const uint32_t hi = (q + 1 >= 0 && q + 1 < n) ? a[q + 1] : 0u;
  return sh == 0 ? lo : (lo >> sh) | (hi << (32 - sh));
}

__global__ void __launch_bounds__(kSeqBitsThreads) tree_bits_seq_kernel(
    const int64_t* __restrict__ parents, long long rows, long long past, long long steps,
    const uint8_t* __restrict__ pad, long long pad_sb, uint32_t* bits, long long row_words, int* first_col,
    unsigned long long* err) {
  extern __shared__ __align__(16) unsigned char seq_smem[];
  const int tw = (int)((rows + 31) / 32);                     // words of a tree bitstring
  long long* par = reinterpret_cast<long long*>(seq_smem);    // [rows]
  uint32_t* prefix = reinterpret_cast<uint32_t*>(par + rows);  // [row_words]
  uint32_t* tree = prefix + row_words;                         // [rows][tw]
  uint32_t* padt = tree + rows * tw;                           // [tw] padding of the tree columns
  const long long b = blockIdx.x;
  const long long cols = past + rows;
  const uint8_t* prow = pad != nullptr ? pad + b * pad_sb : nullptr;
  for (long long i = threadIdx.x; i < rows; i += kSeqBitsThreads) par[i] = parents[b * rows + i];
  for (long long i = threadIdx.x; i < rows * tw; i += kSeqBitsThreads) tree[i] = 0u;
  for (long long i = threadIdx.x; i < tw; i += kSeqBitsThreads) {
    uint32_t word = 0;
    for (int j = 0; j < 32; ++j) {
      const long long t = i * 32 + j;
      if (t < rows && prow != nullptr && prow[past + t]) word |= 1u << j;
    }
    padt[i] = word;
  }
  // prefix: column c <= past is visible unless padded (c == past is the root)
  for (long long w = threadIdx.x; w < row_words; w += kSeqBitsThreads) {
    uint32_t word = 0;
    const long long c0 = w * 32;
    for (int j = 0; j < 32; ++j) {
      const long long c = c0 + j;
      if (c > past) break;
      if (prow == nullptr || !prow[c]) word |= 1u << j;
    }
    prefix[w] = word;
  }
  __syncthreads();
  // ancestors of row r (itself included) within `steps` parent hops
  for (long long r = threadIdx.x; r < rows; r += kSeqBitsThreads) {
    uint32_t* tr = tree + r * tw;
    long long cur = r;
    for (long long k = 0; k < steps; ++k) {
      if (cur >= 0) tr[cur >> 5] |= 1u << (cur & 31);
      const long long at = cur > 0 ? cur : 0;
      if (at >= rows) {
        record_error(err, SPECKV_DERR_TREE_INDEX, at);
        break;
      }
      cur = par[at];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int fc = 0x7f7f7f7f;
    for (long long w = 0; w < row_words; ++w)
      if (prefix[w] != 0u) {
        fc = (int)(w * 32 + __ffs(prefix[w]) - 1);
        break;
      }
    first_col[b] = fc;
  }
  const uint32_t rw = (uint32_t)row_words, total = (uint32_t)(rows * row_words);  // < 2^31: checked on the host
  for (uint32_t idx = threadIdx.x; idx < total; idx += kSeqBitsThreads) {
    const uint32_t r = idx / rw, w = idx - r * rw;
    const long long off = (long long)w * 32 - past;  // tree column offset of the word's first bit
    uint32_t word = prefix[w];
    if (off > -32 && off < rows) word |= bit_window(tree + r * tw, tw, off) & ~bit_window(padt, tw, off);
    if ((long long)w * 32 >= cols) word = 0u;
    bits[b * rows * row_words + idx] = word;
  }
}

// ---------------------------------------------------------------------------
// position / padding update: one warp per sequence.
// ---------------------------------------------------------------------------
__global__ void position_update_kernel(PositionArgs a, long long batch, long long past, long long width,
                                       unsigned long long* err) {
  const long long b = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (b >= batch) return;
  position_row(a, b, past, width, threadIdx.x & 31, err);
}

// ---------------------------------------------------------------------------
// acceptance counters of a round from the packet rows [length, eos?, ...]: one CTA,
// a thread per row (strided), block reduction; writes (does not accumulate) the five sums.
// ---------------------------------------------------------------------------
constexpr int kCountThreads = 256;
__global__ void __launch_bounds__(kCountThreads) acceptance_counts_kernel(const int64_t* __restrict__ packet,
                                                                          long long stride, long long batch,
                                                                          long long proposed, int64_t* counts) {
  __shared__ long long part[kCountThreads / 32][3];
  long long accepted = 0, length = 0, finished = 0;
  for (long long b = threadIdx.x; b < batch; b += kCountThreads) {
    const long long len = packet[b * stride], eos = packet[b * stride + 1];
    accepted += len > 1 ? len - 1 : 0;
    length += len;
    finished += eos != 0;
  }
  for (int o = 16; o > 0; o >>= 1) {
    accepted += __shfl_xor_sync(0xffffffffu, accepted, o);
    length += __shfl_xor_sync(0xffffffffu, length, o);
    finished += __shfl_xor_sync(0xffffffffu, finished, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    part[warp][0] = accepted;
    part[warp][1] = length;
    part[warp][2] = finished;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    long long sums[3] = {0, 0, 0};
    for (int w = 0; w < kCountThreads / 32; ++w)
      for (int k = 0; k < 3; ++k) sums[k] += part[w][k];
    counts[0] = sums[0];
    counts[1] = proposed * batch;
    counts[2] = sums[1];
    counts[3] = batch;
    counts[4] = sums[2];
  }
}

}  // namespace
}  // namespace speckv

using namespace speckv;

extern "C" int speckv_acceptance_counts(const int64_t* packet, int64_t packet_stride_b, int64_t batch,
                                        int64_t proposed_per_row, int64_t* counts, void* stream) {
  const char* fn = "speckv_acceptance_counts";
  if (batch < 0 || proposed_per_row < 0) return fail(SPECKV_EINVAL, "%s: negative size", fn);
  if (batch > 0 && packet_stride_b < 2) return fail(SPECKV_EINVAL, "%s: packet rows need 2 columns", fn);
  if (counts == nullptr || (batch > 0 && packet == nullptr)) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  const int st = check_current_device(fn, {packet, counts});
  if (st) return st;
  acceptance_counts_kernel<<<1, kCountThreads, 0, static_cast<cudaStream_t>(stream)>>>(packet, packet_stride_b,
                                                                                     batch, proposed_per_row, counts);
  return check_launch(fn);
}

extern "C" int speckv_trace_path(const int64_t* parents, const int64_t* tokens, const int64_t* contexts,
                                 const int64_t* samples, int64_t batch, int64_t rows, int64_t eos,
                                 int64_t* out_tokens, int64_t* out_indices, int64_t* out_contexts,
                                 int64_t out_stride_b, int64_t out_stride_w, int64_t width,
                                 int64_t* lengths, void* stream) {
  const char* fn = "speckv_trace_path";
  if (batch < 0 || rows < 1 || width < 0) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (batch == 0) return SPECKV_OK;
  if (!parents || !tokens || !contexts || !samples || !lengths || (width > 0 && (!out_tokens || !out_indices || !out_contexts)))
    return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  const int dst = check_current_device(fn, {samples, lengths});
  if (dst) return dst;
  const int threads = 128;
  const long long blocks = (batch * 32 + threads - 1) / threads;
  trace_path_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      parents, tokens, contexts, samples, batch, rows, eos, out_tokens, out_indices, out_contexts, out_stride_b,
      out_stride_w, width, lengths);
  return check_launch(fn);
}

extern "C" int speckv_pack_tree(const int64_t* full_parents, const int64_t* full_contexts, const int64_t* all_tokens,
                                const int64_t* chosen, int64_t batch, int64_t full_count, int64_t packed_count,
                                int64_t* out_parents, int64_t* out_tokens, int64_t* out_contexts,
                                int64_t out_stride_b, void* stream) {
  const char* fn = "speckv_pack_tree";
  if (batch < 0 || full_count < 0 || packed_count < 0) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (batch == 0) return SPECKV_OK;
  if (!full_parents || !full_contexts || !all_tokens || !out_parents || !out_tokens || !out_contexts ||
      (packed_count > 0 && !chosen))
    return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (full_count + 1 > 50000) return fail(SPECKV_ENOSUPPORT, "%s: %lld draft nodes too many", fn, (long long)full_count);
  const int dst = check_current_device(fn, {full_parents, out_parents});
  if (dst) return dst;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  const size_t smem = (size_t)(full_count + 1) * sizeof(int);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) cudaFuncSetAttribute(pack_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  pack_tree_kernel<<<(unsigned)batch, kPackThreads, smem, s>>>(full_parents, full_contexts, all_tokens, chosen,
                                                               full_count, packed_count, out_parents, out_tokens,
                                                               out_contexts, out_stride_b, err);
  return check_launch(fn);
}

static int launch_pad(const char* fn, PadArgs& a, void* stream) {
  if (a.batch < 0 || a.capacity < 1) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (a.batch == 0) return SPECKV_OK;
  if (a.capacity > (1 << 20)) return fail(SPECKV_ENOSUPPORT, "%s: capacity %lld too large", fn, a.capacity);
  if (!a.tokens || !a.indices || !a.lengths || !a.ot || !a.oi || !a.om || !a.last)
    return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  const int dst = check_current_device(fn, {a.tokens, a.ot, a.packet});
  if (dst) return dst;
  const size_t smem = (size_t)a.capacity * sizeof(int);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) cudaFuncSetAttribute(pad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  pad_kernel<<<(unsigned)a.batch, kPadThreads, smem, s>>>(a);
  return check_launch(fn);
}

extern "C" int speckv_pad_verified_path(const int64_t* tokens, int64_t tok_stride_b, int64_t tok_stride_w,
                                        const int64_t* indices, int64_t idx_stride_b, int64_t idx_stride_w,
                                        const int64_t* lengths, int64_t batch, int64_t capacity,
                                        int64_t width, int64_t past, int64_t eos,
                                        int64_t* out_tokens, int64_t* out_indices, uint8_t* out_mask,
                                        int64_t out_stride_b, int64_t out_stride_w,
                                        int64_t* last, int64_t last_stride, void* stream) {
  const char* fn = "speckv_pad_verified_path";
  if (width < 1 || width > capacity) return fail(SPECKV_EINVAL, "%s: invalid committed path width", fn);
  PadArgs a = {tokens, tok_stride_b, tok_stride_w, indices, idx_stride_b, idx_stride_w, lengths,
               batch, capacity, width, past, eos, out_tokens, out_indices, out_mask, out_stride_b,
               out_stride_w, last, last_stride, nullptr, 0, 0, nullptr};
  return launch_pad(fn, a, stream);
}

extern "C" int speckv_pad_schedule(const int64_t* tokens, int64_t tok_stride_b, int64_t tok_stride_w,
                                   const int64_t* indices, int64_t idx_stride_b, int64_t idx_stride_w,
                                   const int64_t* lengths, int64_t batch, int64_t capacity,
                                   int64_t past, int64_t eos,
                                   int64_t* out_tokens, int64_t* out_indices, uint8_t* out_mask,
                                   int64_t out_stride_b, int64_t out_stride_w,
                                   int64_t* last, int64_t last_stride,
                                   int64_t* packet, int64_t packet_stride_b, int64_t packet_stride_w,
                                   const int64_t* snapshot, void* stream) {
  const char* fn = "speckv_pad_schedule";
  if (packet == nullptr) return fail(SPECKV_EINVAL, "%s: null packet", fn);
  PadArgs a = {tokens, tok_stride_b, tok_stride_w, indices, idx_stride_b, idx_stride_w, lengths,
               batch, capacity, 0, past, eos, out_tokens, out_indices, out_mask, out_stride_b,
               out_stride_w, last, last_stride, packet, packet_stride_b, packet_stride_w, snapshot};
  return launch_pad(fn, a, stream);
}

extern "C" int speckv_tree_mask(const int64_t* parents, int64_t batch, int64_t rows, int64_t past,
                                int64_t steps, void* mask, int32_t dtype, const uint8_t* pad,
                                int64_t pad_stride_b, void* stream) {
  const char* fn = "speckv_tree_mask";
  if (batch < 0 || rows < 1 || past < 0 || steps < 0) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (dtype != SPECKV_F32 && dtype != SPECKV_BF16 && dtype != SPECKV_F16)
    return fail(SPECKV_EINVAL, "%s: unsupported mask dtype %d", fn, dtype);
  if (steps > kMaxSteps) return fail(SPECKV_ENOSUPPORT, "%s: %lld parent hops exceed %d", fn, (long long)steps, kMaxSteps);
  if (batch == 0) return SPECKV_OK;
  if (!parents || !mask) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (batch > 65535) return fail(SPECKV_ENOSUPPORT, "%s: batch above 65535", fn);
  const int dst = check_current_device(fn, {parents, mask, pad});
  if (dst) return dst;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  const long long cols = past + rows;
  const long long chunks = (cols + kMaskCols - 1) / kMaskCols;
  if (chunks > 65535) return fail(SPECKV_ENOSUPPORT, "%s: %lld columns too many", fn, cols);
  dim3 grid((unsigned)rows, (unsigned)batch, (unsigned)chunks);
  tree_mask_kernel<<<grid, kMaskThreads, 0, static_cast<cudaStream_t>(stream)>>>(parents, rows, past, steps, mask,
                                                                                 dtype, pad, pad_stride_b, err);
  return check_launch(fn);
}

extern "C" int speckv_tree_mask_bits(const int64_t* parents, int64_t batch, int64_t rows, int64_t past, int64_t steps,
                                     const uint8_t* pad, int64_t pad_stride_b, uint32_t* bits, int64_t row_words,
                                     int32_t* first_col, void* stream) {
  const char* fn = "speckv_tree_mask_bits";
  if (batch < 0 || rows < 1 || past < 0 || steps < 0) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (steps > kMaxSteps) return fail(SPECKV_ENOSUPPORT, "%s: %lld parent hops exceed %d", fn, (long long)steps, kMaxSteps);
  const long long cols = past + rows;
  if (row_words < 4 * ((cols + 127) / 128))
    return fail(SPECKV_EINVAL, "%s: row_words %lld below 4 * ceil(%lld / 128)", fn, (long long)row_words, cols);
  if (batch == 0) return SPECKV_OK;
  if (!parents || !bits || !first_col) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (batch > 65535) return fail(SPECKV_ENOSUPPORT, "%s: batch above 65535", fn);
  const int dst = check_current_device(fn, {parents, bits, first_col, pad});
  if (dst) return dst;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long tw = (rows + 31) / 32;
  const long long seq_smem = rows * 8 + (row_words + rows * tw + tw) * 4;
  if (rows <= kSeqBitsMaxRows && seq_smem <= 200 * 1024 && rows * row_words < (1ll << 31)) {
    if (seq_smem > 48 * 1024)
      cudaFuncSetAttribute(tree_bits_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)seq_smem);
    tree_bits_seq_kernel<<<(unsigned)batch, kSeqBitsThreads, (size_t)seq_smem, s>>>(
        parents, rows, past, steps, pad, pad_stride_b, bits, row_words, first_col, err);
    return check_launch(fn);
  }
  // 0x7f7f7f7f: larger than any column, lowered by atomicMin in the kernel
  cudaError_t e = cudaMemsetAsync(first_col, 0x7f, (size_t)batch * sizeof(int32_t), s);
  if (e != cudaSuccess) return fail(SPECKV_ECUDA, "%s: %s", fn, cudaGetErrorString(e));
  dim3 grid((unsigned)rows, (unsigned)batch);
  tree_bits_kernel<<<grid, kMaskThreads, 0, s>>>(parents, rows, past, steps, pad, pad_stride_b, bits, row_words,
                                                 first_col, err);
  return check_launch(fn);
}

extern "C" int speckv_position_update(uint8_t* pad_rows, int64_t pad_rows_stride, int64_t pad_rows_count,
                                      const int64_t* owners, uint8_t* pad_live, int64_t pad_live_stride,
                                      const uint8_t* newly_padded, int64_t np_stride_b, int64_t batch,
                                      int64_t past, int64_t width, int64_t* positions,
                                      int64_t positions_stride_b, int64_t* past_positions, void* stream) {
  const char* fn = "speckv_position_update";
  if (batch < 0 || past < 0 || width < 1) return fail(SPECKV_EINVAL, "%s: bad sizes", fn);
  if (batch == 0) return SPECKV_OK;
  if (!newly_padded || !positions || !past_positions) return fail(SPECKV_EINVAL, "%s: null pointer", fn);
  if (pad_rows != nullptr && (owners == nullptr || past + width > pad_rows_stride))
    return fail(SPECKV_EINVAL, "%s: padding rows need owners and past + width <= row stride", fn);
  if (pad_live != nullptr && past + width > pad_live_stride)
    return fail(SPECKV_EINVAL, "%s: past + width exceeds live padding row stride", fn);
  const int dst = check_current_device(fn, {newly_padded, positions, pad_rows});
  if (dst) return dst;
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "%s: device error word unavailable", fn);
  const int threads = 128;
  const long long blocks = (batch * 32 + threads - 1) / threads;
  const PositionArgs a{pad_rows, pad_rows_stride, pad_rows_count, owners, pad_live, pad_live_stride,
                       newly_padded, np_stride_b, positions, positions_stride_b, past_positions};
  position_update_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(a, batch, past, width,
                                                                                            err);
  return check_launch(fn);
}
