// Tree-verify GQA attention on Blackwell tensor cores (sm_100a): tcgen05.mma
// with TMEM accumulators, K/V tiles streamed by TMA (no multicast), warp
// specialised.
//
// Work unit (one CTA): sequence b, KV head h, and a tile of 128 "packed rows".
// The g = q_heads / kv_heads query heads that share KV head h are packed with
// the tree rows into one M dimension, row m = r * g + j (tree row r, head
// h * g + j), so K/V of (b, h) stream once for all of them (no repeat_kv).
//
//   warp 0      TMA producer: K and V tiles (128 positions x 128 dims, bf16/fp16,
//               128-byte swizzle) into a 2-stage ring
//   warp 1      TMEM owner + MMA issuer (one thread): S = Q K^T into a double
//               buffered TMEM S, then O += P V into TMEM O
//   warps 4-7   softmax: thread t owns row t (TMEM lane t); reads S with
//               tcgen05.ld, masks, online softmax in the log2 domain with lazy
//               rescaling of O, writes P (bf16/fp16) to shared memory; epilogue
//               normalises O and stores it.
//
// Visibility comes either from a bit-packed (batch, rows, words) mask built
// once per verify round (BITS mode) or from a dense additive mask (DENSE mode,
// the drop-in path). Left-padding tiles are skipped via first_col[b].
//
// Every mbarrier wait is bounded (about 2 s of %globaltimer); on expiry the
// kernel records SPECKV_DERR_TIMEOUT in the device error word and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "attention.cuh"
#include "common.cuh"

namespace speckv {
namespace {

constexpr int BM = 128;   // packed rows per CTA (TMEM lanes)
constexpr int BN = 128;   // key positions per tile
constexpr int HD = 128;   // head dim
constexpr int kStages = 2;
constexpr int kThreads = 256;
constexpr uint32_t kTileHalf = BM * 128;         // 16 KB: 128 rows x 64 elements x 2 B
constexpr uint32_t kTileBytes = 2 * kTileHalf;   // 32 KB: 128 rows x 128 elements
constexpr uint32_t Q_OFF = 0;
constexpr uint32_t KV_OFF = Q_OFF + kTileBytes;
constexpr uint32_t STAGE_BYTES = 2 * kTileBytes;  // K + V
constexpr uint32_t P_OFF = KV_OFF + kStages * STAGE_BYTES;
constexpr uint32_t BAR_OFF = P_OFF + kTileBytes;
constexpr uint32_t SMEM_BYTES = BAR_OFF + 256 + 1024;  // + barriers + alignment slack
// Staged dense mask (MODE 2): warps 2-3 copy the mask rows of the CTA's 128 packed rows
// (at most 127 / g + 2 tree rows) for each key tile into a 2-stage shared-memory ring, all
// loads of a tile in flight at once; rows padded by 16 bytes so the softmax warps' row reads
// fall in distinct banks. Query groups g >= 4 (16-bit masks) or g >= 5 (fp32 masks).
constexpr uint32_t MASK_OFF = BAR_OFF + 256;
template <typename MT>
__host__ __device__ constexpr int mask_cta_rows() { return sizeof(MT) == 4 ? 27 : 33; }
template <typename MT>
__host__ __device__ constexpr int mask_min_group() { return sizeof(MT) == 4 ? 5 : 4; }
template <typename MT>
__host__ __device__ constexpr uint32_t mask_row_bytes() { return BN * (uint32_t)sizeof(MT) + 16u; }
template <typename MT>
__host__ __device__ constexpr uint32_t mask_stage_bytes() { return mask_cta_rows<MT>() * mask_row_bytes<MT>(); }
static_assert(127 / 4 + 2 <= 33 && 127 / 5 + 2 <= 27, "a CTA's tree rows must fit its mask stage");
static_assert(SMEM_BYTES + 2 * mask_stage_bytes<float>() <= 232448 &&
              SMEM_BYTES + 2 * mask_stage_bytes<uint16_t>() <= 232448, "staged mask exceeds shared memory");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t S_COL0 = 0, O_COL = 256;
constexpr unsigned long long kWaitNs = 2000000000ull;

// Test hooks (speckv_attention_test_hooks): a shorter limit for the bounded waits
// (0 = kWaitNs) and a switch that makes CTA 0's first softmax warpgroup withhold its
// first Q-tile arrival, so that the MMA warp's wait runs out with no copy or MMA in
// flight. Both stay 0 in normal use; they are read only on the slow path of a wait
// and once per CTA.
__device__ unsigned long long g_wait_limit_ns = 0ull;
__device__ int g_withhold_q_arrival = 0;

// Key-range chunks (the pair kernel's CHUNKS form): when a sequence has more key tiles than a
// CTA's average share of the launch, its items are split into chunks of about that share, and
// each chunk leaves its partial result here: per launch slot, a merge counter per (sequence,
// KV head, row tile) and the partial tiles, 128 rows of 128 unnormalised O values plus the
// running max and sum (fp32, rows padded to 132 floats). The warpgroup that finishes a row
// tile's last chunk merges the partials, writes the output and zeroes the counter; launches
// that may run at the same time take different slots.
constexpr int kPartSlots = 4;
constexpr int kPartCounters = 1 << 16;
constexpr int kPartTiles = 240;
constexpr int kPartRowFloats = 132;
constexpr int kPartTileFloats = 128 * kPartRowFloats;
constexpr int kMaxChunks = 8;
__device__ int g_part_count[kPartSlots * kPartCounters];
__device__ __align__(16) float g_part[(size_t)kPartSlots * kPartTiles * kPartTileFloats];

__device__ __forceinline__ unsigned long long wait_limit() {
  const unsigned long long v = *reinterpret_cast<volatile unsigned long long*>(&g_wait_limit_ns);
  return v != 0ull ? v : kWaitNs;
}

// barrier slots (8 bytes each) after BAR_OFF
enum { B_KV_FULL = 0, B_KV_EMPTY = 2, B_S_FULL = 4, B_S_FREE = 6, B_P_FULL = 8, B_O_DONE = 9, B_Q_READY = 10,
       B_DRAIN = 11, B_ABORT = 12, TMEM_SLOT = 13, B_M_FULL = 14, B_M_EMPTY = 16 };

struct Sm100Args {
  const void* q;
  long long qs0, qs1, qs2;
  void* out;
  const uint32_t* bits;   // BITS mode: (batch, rows, row_words)
  long long row_words;
  const int* first_col;   // BITS mode (optional)
  const void* mask;       // DENSE mode: (batch, 1, rows, kv_len)
  int mask_dtype;
  int batch, q_heads, kv_heads, group, rows, kv_len, mtiles;
  float scale_log2;       // softmax scale * log2(e)
  int part_slot;          // pair kernel with key-range chunks: slot of this launch's partials
  int past;               // pair kernel with the append fused: cached positions before the tree rows
  unsigned long long* err;
};

// The append fused into the pair kernel: the round's new K / V rows ((batch, KV heads, rows,
// 128) strided views, read as each sequence's last key tile) and the pools they are stored
// into at position `past` (maps over the first past + rows positions, so a 128-row store box
// writes exactly the new rows). Unused by the other instantiations.
struct AppendMaps {
  CUtensorMap k_new, v_new, k_pool, v_pool;
};

// K/V rows of each sequence for the pair kernel (NULL map: sequence b is row b); a separate
// kernel argument so the table-free kernels' argument block stays as it was.
struct KvRows {
  const int64_t* map;
  int rows;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait; returns false (and records a timeout) if the phase never completes
// or another role already gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long* err, int where) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns(), limit = wait_limit();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > limit) {
        *abort_flag = 1;
        record_error(err, SPECKV_DERR_TIMEOUT, where);
        return false;
      }
    }
  }
}

// Time-bounded wait that ignores the abort flag: used to let in-flight asynchronous
// work finish before the CTA releases shared memory / TMEM. It keeps the full limit
// (never the test hook's shorter one): copies in flight must land.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try(bar, parity)) {
    if (global_ns() - t0 > kWaitNs) return;
  }
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// L2 prefetch of one box of a tensor map (no shared-memory destination, no barrier).
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

// TMA store of one box from shared memory (bulk-group completion, no barrier); the caller
// commits the group and waits for its reads before the shared memory is reused.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// The low n bits of a visibility word (n <= 0: none, n >= 32: all).
__device__ __forceinline__ uint32_t low_bits(int n) { return n >= 32 ? 0xffffffffu : n <= 0 ? 0u : (1u << n) - 1u; }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (thread t <- lane base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  uint32_t r[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format: version 1 at bits 46-47,
// layout type 2 at bits 61-63). lbo / sbo in bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: f32 accumulate, A/B type (0 f16, 1 bf16), K-major A,
// B major (0 K, 1 MN), N = 128, M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t ab_type, uint32_t b_mn_major) {
  return (1u << 4) | (ab_type << 7) | (ab_type << 10) | (b_mn_major << 16) | ((uint32_t)(HD >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

template <typename T> struct TypeCode;
template <> struct TypeCode<__nv_bfloat16> { static constexpr uint32_t value = 1; };
template <> struct TypeCode<__half> { static constexpr uint32_t value = 0; };

// byte offset of 16-byte chunk `c` (0..15) of row `m` in a [2][128 rows][128 B] swizzled tile
__device__ __forceinline__ uint32_t sw_chunk(uint32_t m, uint32_t c) {
  return (c >> 3) * kTileHalf + m * 128u + (((c & 7u) ^ (m & 7u)) << 4);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}

template <typename M>
__device__ __forceinline__ float mask_value(const void* mask, long long idx);
template <>
__device__ __forceinline__ float mask_value<float>(const void* mask, long long idx) {
  return static_cast<const float*>(mask)[idx];
}
template <>
__device__ __forceinline__ float mask_value<__nv_bfloat16>(const void* mask, long long idx) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(mask)[idx]);
}
template <>
__device__ __forceinline__ float mask_value<__half>(const void* mask, long long idx) {
  return __half2float(static_cast<const __half*>(mask)[idx]);
}

// raw bits of one mask element and their float value
template <typename MT> struct MaskRaw { using type = uint16_t; };
template <> struct MaskRaw<float> { using type = uint32_t; };
template <typename MT>
__device__ __forceinline__ float mask_raw_value(uint32_t raw);
template <>
__device__ __forceinline__ float mask_raw_value<float>(uint32_t raw) { return __uint_as_float(raw); }
template <>
__device__ __forceinline__ float mask_raw_value<__nv_bfloat16>(uint32_t raw) { return __uint_as_float(raw << 16); }
template <>
__device__ __forceinline__ float mask_raw_value<__half>(uint32_t raw) {
  return __half2float(__ushort_as_half((unsigned short)raw));
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
// MODE 0: visibility bits; MODE 1: dense additive mask of type MT read per thread from
// global memory; MODE 2: the same mask staged in shared memory by warps 2-3.
template <typename T, int MODE, typename MT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_sm100_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      const Sm100Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + BAR_OFF;
  auto bar = [&](int i) { return bar0 + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + BAR_OFF + 8 * B_ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BAR_OFF + 8 * TMEM_SLOT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x % a.mtiles;
  const int bh = blockIdx.x / a.mtiles;
  const int b = bh / a.kv_heads, kvh = bh % a.kv_heads;
  const int total_rows = a.group * a.rows;
  const int n_tiles_all = (a.kv_len + BN - 1) / BN;
  int tile0 = 0;
  if (MODE == 0 && a.first_col != nullptr) {
    const int fc = a.first_col[b];
    tile0 = fc < 0 ? 0 : min(fc / BN, n_tiles_all - 1);
  }
  const int n_tiles = n_tiles_all - tile0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_KV_FULL + i), 1);
      mbar_init(bar(B_KV_EMPTY + i), 1);
      mbar_init(bar(B_S_FULL + i), 1);
      mbar_init(bar(B_S_FREE + i), 128);
      mbar_init(bar(B_M_FULL + i), 64);
      mbar_init(bar(B_M_EMPTY + i), 128);
    }
    mbar_init(bar(B_P_FULL), 128);
    mbar_init(bar(B_O_DONE), 1);
    mbar_init(bar(B_Q_READY), 128);
    mbar_init(bar(B_DRAIN), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
      int issued = 0;
      for (int it = 0; it < n_tiles; ++it) {
        const int s = it & 1;
        if (it >= 2 && !mbar_wait(bar(B_KV_EMPTY + s), ((it >> 1) - 1) & 1, abort_flag, a.err, 1)) break;
        issued = it + 1;
        const uint32_t kdst = sbase + KV_OFF + s * STAGE_BYTES;
        const uint32_t vdst = kdst + kTileBytes;
        const int col = (tile0 + it) * BN;
        mbar_expect_tx(bar(B_KV_FULL + s), STAGE_BYTES);
        tma_load_4d(kdst, &tmk, bar(B_KV_FULL + s), 0, col, kvh, b);
        tma_load_4d(kdst + kTileHalf, &tmk, bar(B_KV_FULL + s), 64, col, kvh, b);
        tma_load_4d(vdst, &tmv, bar(B_KV_FULL + s), 0, col, kvh, b);
        tma_load_4d(vdst + kTileHalf, &tmv, bar(B_KV_FULL + s), 64, col, kvh, b);
      }
      // Copies still in flight must land before shared memory is released: after an abort
      // nobody consumes them (in a normal run these phases completed long ago).
      for (int it = issued - 2 < 0 ? 0 : issued - 2; it < issued; ++it) drain_wait(bar(B_KV_FULL + (it & 1)), (it >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t ab = TypeCode<T>::value;
      const uint32_t id_s = idesc_f16(ab, 0), id_pv = idesc_f16(ab, 1);
      const uint32_t o_tmem = tmem + O_COL;
      bool ok = mbar_wait(bar(B_Q_READY), 0, abort_flag, a.err, 3);
      tc_fence_after();
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(bar(B_P_FULL), j & 1, abort_flag, a.err, 4)) return false;
        tc_fence_after();
        const uint32_t vbase = sbase + KV_OFF + (j & 1) * STAGE_BYTES + kTileBytes;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sw128_desc(sbase + P_OFF + (kk >> 2) * kTileHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(vbase + kk * 2048, kTileHalf, 1024);
          tc_mma(o_tmem, ad, bd, id_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar(B_O_DONE));
        tc_commit(bar(B_KV_EMPTY + (j & 1)));
        return true;
      };
      for (int it = 0; ok && it < n_tiles; ++it) {
        const int s = it & 1;
        if (!mbar_wait(bar(B_KV_FULL + s), (it >> 1) & 1, abort_flag, a.err, 5)) { ok = false; break; }
        if (it >= 2 && !mbar_wait(bar(B_S_FREE + s), ((it >> 1) - 1) & 1, abort_flag, a.err, 6)) { ok = false; break; }
        tc_fence_after();
        const uint32_t kbase = sbase + KV_OFF + s * STAGE_BYTES;
        const uint32_t s_tmem = tmem + S_COL0 + s * BN;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t ad = sw128_desc(sbase + Q_OFF + (kk >> 2) * kTileHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(kbase + (kk >> 2) * kTileHalf + (kk & 3) * 32, 16, 1024);
          tc_mma(s_tmem, ad, bd, id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(bar(B_S_FULL + s));
        if (it >= 1 && !issue_pv(it - 1)) { ok = false; break; }
      }
      if (ok && n_tiles > 0) issue_pv(n_tiles - 1);
      // every MMA issued by this thread completes before TMEM is released
      tc_commit(bar(B_DRAIN));
      drain_wait(bar(B_DRAIN), 0);
    }
  } else if (MODE == 2 && warp < 4) {
    // ---------------- mask loader (warps 2-3) ----------------
    using Raw = typename MaskRaw<MT>::type;
    constexpr int kLoads = 2 * mask_cta_rows<MT>();  // per thread: 64 threads x kLoads >= rows x 128
    const int lt = threadIdx.x - 64;
    const int r_lo = (mt * BM) / a.group;
    const int nr = (min(total_rows, mt * BM + BM) - 1) / a.group - r_lo + 1;
    const Raw* src = static_cast<const Raw*>(a.mask) + ((long long)b * a.rows + r_lo) * a.kv_len;
    for (int it = 0; it < n_tiles; ++it) {
      const int s = it & 1;
      if (it >= 2 && !mbar_wait(bar(B_M_EMPTY + s), ((it >> 1) - 1) & 1, abort_flag, a.err, 11)) break;
      const int c0 = (tile0 + it) * BN;
      // element u of this thread: row u / 2, column (u % 2) * 64 + lt of the tile
      Raw v[kLoads];
#pragma unroll
      for (int u = 0; u < kLoads; ++u) {
        const int rr = u >> 1, c = (u & 1) * 64 + lt;
        v[u] = (rr < nr && c0 + c < a.kv_len) ? __ldg(src + (long long)rr * a.kv_len + c0 + c) : Raw(0);
      }
      uint8_t* dst = smem + MASK_OFF + s * mask_stage_bytes<MT>();
#pragma unroll
      for (int u = 0; u < kLoads; ++u) {
        const int rr = u >> 1, c = (u & 1) * 64 + lt;
        if (rr < nr) *reinterpret_cast<Raw*>(dst + rr * mask_row_bytes<MT>() + c * sizeof(Raw)) = v[u];
      }
      mbar_arrive(bar(B_M_FULL + s));
    }
  } else if (warp >= 4) {
    // ---------------- softmax warpgroup ----------------
    const int t = threadIdx.x - 128;  // row within the tile == TMEM lane
    const int quarter = warp & 3;     // TMEM lane quarter this warp may access
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int grow = mt * BM + t;     // packed row
    const bool valid = grow < total_rows;
    const int r = valid ? grow / a.group : 0;
    const int hq = kvh * a.group + (valid ? grow % a.group : 0);
    // Q row -> swizzled shared tile (zeros for padding rows)
    {
      const T* qrow = static_cast<const T*>(a.q) + (long long)b * a.qs0 + (long long)hq * a.qs1 + (long long)r * a.qs2;
      uint4 v[16];  // all loads in flight before the first shared-memory store
#pragma unroll
      for (int c = 0; c < 16; ++c) v[c] = valid ? __ldg(reinterpret_cast<const uint4*>(qrow) + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < 16; ++c) *reinterpret_cast<uint4*>(smem + Q_OFF + sw_chunk(t, c)) = v[c];
      fence_proxy_async();
      mbar_arrive(bar(B_Q_READY));
    }
    using Raw = typename MaskRaw<MT>::type;
    const int r_lo = (mt * BM) / a.group;  // MODE 2: first tree row of the staged mask rows
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int it = 0; it < n_tiles; ++it) {
      const int s = it & 1;
      ok = mbar_wait(bar(B_S_FULL + s), (it >> 1) & 1, abort_flag, a.err, 7);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float x[BN];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_addr + S_COL0 + s * BN + c * 32, x + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar(B_S_FREE + s));  // S buffer may take S of tile it + 2
      const int col0 = (tile0 + it) * BN;
      float mx = -INFINITY;
      if (MODE == 0) {
        uint4 w = make_uint4(0, 0, 0, 0);
        if (valid) w = *reinterpret_cast<const uint4*>(a.bits + ((long long)b * a.rows + r) * a.row_words + (tile0 + it) * 4);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const bool vis = (words[i >> 5] >> (i & 31)) & 1u;
          x[i] = vis ? x[i] * a.scale_log2 : -INFINITY;
          mx = fmaxf(mx, x[i]);
        }
      } else if (MODE == 2) {
        ok = mbar_wait(bar(B_M_FULL + s), (it >> 1) & 1, abort_flag, a.err, 10);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        const uint8_t* mrow = smem + MASK_OFF + s * mask_stage_bytes<MT>() + (valid ? r - r_lo : 0) * mask_row_bytes<MT>();
        constexpr float kLog2e = 1.4426950408889634f;
        constexpr int kPer = 16 / (int)sizeof(Raw);
#pragma unroll
        for (int i0 = 0; i0 < BN; i0 += kPer) {
          const uint4 w = *reinterpret_cast<const uint4*>(mrow + i0 * sizeof(Raw));
          const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < kPer; ++j) {
            const uint32_t raw = sizeof(Raw) == 4 ? wv[j] : (wv[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
            const int i = i0 + j;
            x[i] = col0 + i < a.kv_len ? x[i] * a.scale_log2 + mask_raw_value<MT>(raw) * kLog2e : -INFINITY;
            mx = fmaxf(mx, x[i]);
          }
          // at most four 16-byte reads in flight: keeps fp32 masks within the register budget
          if (sizeof(Raw) == 4 && (i0 / kPer) % 4 == 3) asm volatile("" ::: "memory");
        }
        mbar_arrive(bar(B_M_EMPTY + s));  // stage s may take the rows of tile it + 2
      } else {
        const long long mrow = ((long long)b * a.rows + r) * a.kv_len;
        constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int col = col0 + i;
          if (col < a.kv_len) {
            const float mv = a.mask != nullptr ? mask_value<MT>(a.mask, mrow + col) : 0.f;
            x[i] = x[i] * a.scale_log2 + mv * kLog2e;
          } else {
            x[i] = -INFINITY;
          }
          mx = fmaxf(mx, x[i]);
        }
      }
      // lazy rescale: move the running max only when it grows by more than 2^8
      const bool grow_max = mx > m_run + 8.0f;
      const float m_new = grow_max ? mx : m_run;
      const float corr = (grow_max && m_run != -INFINITY) ? ex2(m_run - m_new) : 1.f;
      if (it > 0) {
        // O of the previous tiles must be final before rescaling it or overwriting P
        ok = mbar_wait(bar(B_O_DONE), (it - 1) & 1, abort_flag, a.err, 8);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_addr + O_COL + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(tmem + lane_addr + O_COL + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      m_run = m_new;
      const float base = m_run == -INFINITY ? 0.f : m_run;
      float sum = 0.f;
      uint8_t* prow = smem + P_OFF;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          p[i] = ex2(x[c * 8 + i] - base);
          sum += p[i];
        }
        uint4 v;
        v.x = pack2<T>(p[0], p[1]);
        v.y = pack2<T>(p[2], p[3]);
        v.z = pack2<T>(p[4], p[5]);
        v.w = pack2<T>(p[6], p[7]);
        *reinterpret_cast<uint4*>(prow + sw_chunk(t, c)) = v;
      }
      l_run = l_run * corr + sum;
      tc_fence_before();
      fence_proxy_async();
      mbar_arrive(bar(B_P_FULL));
    }
    if (ok && n_tiles > 0) ok = mbar_wait(bar(B_O_DONE), (n_tiles - 1) & 1, abort_flag, a.err, 9);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* orow = static_cast<T*>(a.out) + (((long long)b * a.rows + r) * a.q_heads + hq) * HD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_addr + O_COL + c * 32, o);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = pack2<T>(o[i] * inv, o[i + 1] * inv);
            v.y = pack2<T>(o[i + 2] * inv, o[i + 3] * inv);
            v.z = pack2<T>(o[i + 4] * inv, o[i + 5] * inv);
            v.w = pack2<T>(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Two-tile persistent kernel (visibility bits). One CTA per SM walks a
// longest-first list of work items (sequence b, KV head, pair of 128-row tiles);
// both row tiles of an item consume every K/V tile it loads.
//
// Row packing: a 128-row tile holds q = floor(128 / g) whole tree rows, tile row
// s = (r - q * tile) * g + j for tree row r and query head j of the KV group, so
// that one 4-D TMA box (64 dims x g heads x q rows) fetches it from the strided
// projection; rows q * g .. 127 stay zero (they are never written).
//
//   warp 3      TMA producer of the Q tiles: the next item's, as soon as the last S
//               MMA of the current item has read the Q buffer
//   warp 0      TMA producer of the K tiles (2-stage ring); prefetches the next item's
//               first tiles into L2
//   warp 2      TMA producer of the V tiles (2-stage ring)
//   warp 1      TMEM owner (512 columns: S0 | S1 | O0 | O1) + MMA issuer, order per
//               key tile i: S0_i, P1_{i-1} V_{i-1}, S1_i, P0_i V_i, so each softmax
//               warpgroup works while the tensor pipe serves the other tile
//   warps 4-7   softmax of row tile 0; warps 8-11 softmax of row tile 1: thread =
//               row = TMEM lane (warp % 4 picks the lane quarter); S is read once
//               into registers, P (16-bit) goes back into the first 64 columns of
//               its S buffer and feeds the P.V MMA straight from TMEM.
// A tcgen05.commit covers every earlier MMA of the issuing thread, so when a
// softmax warpgroup sees S_t,i complete, P_t,i-1 . V_i-1 has finished too: O_t
// may be rescaled and the P region rewritten without further waits.
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 384;
// Register split after the prologue (setmaxnreg): the producer / MMA warpgroup drops
// to kRegsLow, the two softmax warpgroups rise to kRegsHigh. The block is launched
// with kRegsLaunch per thread (the host checks the compiled count), and
// 128 * kRegsLow + 256 * kRegsHigh == 384 * kRegsLaunch, so every increase is
// covered by the decrease. 88 / 208 leaves the softmax loop (128 scores per thread)
// almost free of spills; below 88 the producer and MMA warps spill instead.
constexpr int kRegsLaunch = 168, kRegsLow = 88, kRegsHigh = 208;
static_assert(128 * kRegsLow + 256 * kRegsHigh == kThreads2 * kRegsLaunch, "register split must balance");
constexpr int kMaxSortB = 1024;
constexpr uint32_t Q2_OFF = 0;                    // Q tile t at Q2_OFF + t * kTileBytes
constexpr uint32_t K2_OFF = 2 * kTileBytes;       // K stage s at K2_OFF + s * kTileBytes
constexpr uint32_t V2_OFF = 4 * kTileBytes;       // V stage s at V2_OFF + s * kTileBytes
constexpr uint32_t KEY2_OFF = 6 * kTileBytes;     // int keys[kMaxSortB]
constexpr uint32_t ORD2_OFF = KEY2_OFF + 4 * kMaxSortB;  // int order[kMaxSortB]
constexpr uint32_t BAR2_OFF = ORD2_OFF + 4 * kMaxSortB;
constexpr uint32_t SMEM2_BYTES = BAR2_OFF + 256 + 1024;
// the CHUNKS form adds, past the end of the common layout: start[kMaxSortB + 2] (first item of
// each rank), pbase[kMaxSortB] (first partial tile of each sequence), cinfo[kMaxSortB] (chunk
// length | chunk count << 16 of each sequence)
constexpr uint32_t START2_OFF = BAR2_OFF + 256;
constexpr uint32_t PBASE2_OFF = START2_OFF + 4 * (kMaxSortB + 2);
constexpr uint32_t CINFO2_OFF = PBASE2_OFF + 4 * kMaxSortB;
constexpr uint32_t SMEM2C_BYTES = CINFO2_OFF + 4 * kMaxSortB + 1024;
static_assert(SMEM2C_BYTES <= 232448, "shared memory of the CHUNKS form");
__host__ __device__ constexpr uint32_t S_COL(int t) { return (uint32_t)t * 128u; }
__host__ __device__ constexpr uint32_t O2_COL(int t) { return 256u + (uint32_t)t * 128u; }

enum { C_K_FULL = 0, C_K_EMPTY = 2, C_V_FULL = 4, C_V_EMPTY = 6, C_S_FULL = 8, C_O_FINAL = 10, C_Q_FULL = 12,
       C_P_FULL = 14, C_DRAIN = 16, C_ABORT = 17, C_TMEM_SLOT = 18, C_XCHG = 19, C_Q_EMPTY = 20, C_O_READ = 22,
       C_PH_FULL = 24, C_PLAN = 26, C_LAST = 28 };
static_assert(8 * (C_LAST + 1) <= 256, "barrier area");

// Key-range split of a sequence of n key tiles for a target of `avg` tiles per chunk: the
// chunk length and the number of (non-empty) chunks.
__host__ __device__ inline void split_of(int n, int avg, int& len, int& nch) {
  int n0 = n > avg ? (n + avg - 1) / avg : 1;
  n0 = n0 < kMaxChunks ? n0 : kMaxChunks;
  len = (n + n0 - 1) / n0;
  nch = (n + len - 1) / len;
}

// Warp-wide forms: every lane runs the same code (the operands stay warp-uniform) and
// one elected lane, always lane 0 with the full mask, issues the instruction; the
// commits are issued by that same lane, so they track its MMAs.
__device__ __forceinline__ void tc_mma_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n .reg .b32 r;\n elect.sync r|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n .reg .b32 r;\n elect.sync r|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// true on one lane of the (converged) warp, the same lane every time with the full mask
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile("{\n .reg .pred p;\n .reg .b32 r;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ void tc_commit_w(uint32_t bar) {
  asm volatile(
      "{\n .reg .pred e;\n .reg .b32 r;\n elect.sync r|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 bytes to global memory in one instruction (address 32-byte aligned)
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// (a.x * b.x + c.x, a.y * b.y + c.y) and (a.x + b.x, a.y + b.y) on the packed f32x2 pipe
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long ra, rb, rc, rd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(rd));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long ra, rb, rd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(rd));
  return d;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair on the FMA pipe (relieves the MUFU ex2 unit, which alone would
// bound the softmax): x = n + f with n = rint(x) from the 1.5 * 2^23 shift, 2^f by a
// degree-3 polynomial on [-0.5, 0.5] (minimax in relative error, fitted by linear
// programming on 2049 points; max relative error 7.5e-5, below the 16-bit rounding
// of P), and 2^n applied as one multiply by the float whose exponent field is n + 127.
// x <= -127 (masked scores are -inf) gives exactly +0. Valid for x < 128; larger
// arguments only occur in a tile that is recomputed against a larger reference.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float2 xc = make_float2(fmaxf(x.x, -127.f), fmaxf(x.y, -127.f));
  const float2 t = __fadd2_rn(xc, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __fadd2_rn(xc, make_float2(-n.x, -n.y));
  float2 p = __ffma2_rn(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.2426111251f, 0.2426111251f));
  p = __ffma2_rn(p, f, make_float2(0.6932609678f, 0.6932609678f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  // bits(t) = 0x4B400000 + n, so (bits(t) + 127) << 23 == (n + 127) << 23 (mod 2^32): 2^n,
  // and exactly 0 for n = -127
  const float sx = __uint_as_float((__float_as_uint(t.x) + 127u) << 23);
  const float sy = __uint_as_float((__float_as_uint(t.y) + 127u) << 23);
  return __fmul2_rn(p, make_float2(sx, sy));
}

// Which 2-column pairs take the polynomial (1 in 4): moves a quarter of the exponentials
// from the MUFU unit (16 results per clock per SM) to the FMA pipe (~15 issue slots per
// pair); the measured optimum between all-MUFU and half-and-half.
__host__ __device__ constexpr bool poly_pair(int q) { return (q & 7) == 1 || (q & 7) == 5; }

struct Item {
  int b, kvh, pair;  // CHUNKS: pair holds the row-tile pair in bits 0-15 and the key-range chunk above
};

// SPLIT (at most 128 packed rows per (sequence, KV head), e.g. a draft step): both
// softmax warpgroups serve the one Q tile and take alternate key tiles (warpgroup w the
// tiles i with i % 2 == w); S_w of tile i and the P.V of tile i - 1 are issued in turn,
// so the K and V rings are consumed in order. Warpgroup 1 hands its running max and sum
// to warpgroup 0 through shared memory (C_XCHG, a bounded wait), which merges O0 and O1
// and then signals C_O_READ: the next item's first P.V waits for it.
// TABLE: the K/V rows of sequence b come from a.row_table[b] (a separate instantiation, so
// the table-free kernel carries no trace of it).
// APPEND: the round's tree rows are appended by this launch. The key tiles are the cached
// positions [0, past) in 128-key tiles (tmk / tmv cover only those positions, so the last,
// partial tile reads zeros past them), then one tree tile [past, past + rows) loaded from
// the new rows (am.k_new / am.v_new). The producer of the item holding row-tile pair 0 of
// a (sequence, KV head) stores that tile into the pools at position past once it has
// landed (TMA store from the K / V ring stage, waited for before the stage is refilled).
// Visibility of the partial tile is cut at past; the tree tile's words start at bit past.
template <typename T, bool SPLIT, bool TABLE, bool CHUNKS, bool APPEND = false>
__global__ void __launch_bounds__(kThreads2, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const __grid_constant__ CUtensorMap tmq, const Sm100Args a, const KvRows kvr,
                     const __grid_constant__ AppendMaps am) {
  static_assert(!APPEND || (!TABLE && !CHUNKS), "the fused append runs without row tables and key-range chunks");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + BAR2_OFF;
  auto bar = [&](int i) { return bar0 + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + BAR2_OFF + 8 * C_ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BAR2_OFF + 8 * C_TMEM_SLOT);
  int* keys = reinterpret_cast<int*>(smem + KEY2_OFF);
  int* order = reinterpret_cast<int*>(smem + ORD2_OFF);
  // CHUNKS only (unused otherwise)
  int* start = reinterpret_cast<int*>(smem + START2_OFF);
  int* pbase = reinterpret_cast<int*>(smem + PBASE2_OFF);
  int* cinfo = reinterpret_cast<int*>(smem + CINFO2_OFF);
  int* plan = reinterpret_cast<int*>(smem + BAR2_OFF + 8 * C_PLAN);  // tile sum, tile maximum
  volatile int* lastf = reinterpret_cast<volatile int*>(smem + BAR2_OFF + 8 * C_LAST);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qrows = BM / a.group;                        // whole tree rows per 128-row tile
  const int mtiles = (a.rows + qrows - 1) / qrows;       // row tiles per (sequence, KV head)
  const int pairs = SPLIT ? 1 : (mtiles + 1) / 2;
  const int per_b = a.kv_heads * pairs;
  int n_items = a.batch * per_b;
  // APPEND: cached tiles [0, n_cached), then the tree tile n_cached
  const int n_cached = APPEND ? (a.past + BN - 1) / BN : 0;
  const int n_tiles_all = APPEND ? n_cached + 1 : (a.kv_len + BN - 1) / BN;
  const bool sorted = a.batch <= kMaxSortB;
  auto first_tile = [&](int b) {
    if (a.first_col == nullptr) return 0;
    const int fc = a.first_col[b];
    return fc < 0 ? 0 : min(fc / BN, n_tiles_all - 1);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(C_K_FULL + i), 1);
      mbar_init(bar(C_K_EMPTY + i), 1);
      mbar_init(bar(C_V_FULL + i), 1);
      mbar_init(bar(C_V_EMPTY + i), 1);
      mbar_init(bar(C_S_FULL + i), 1);
      mbar_init(bar(C_O_FINAL + i), 1);
      mbar_init(bar(C_Q_FULL + i), 1);
      mbar_init(bar(C_Q_EMPTY + i), 1);
      mbar_init(bar(C_P_FULL + i), 128);
      mbar_init(bar(C_PH_FULL + i), 128);
    }
    if (CHUNKS) {  // tile sum and maximum over the sequences, accumulated by the sort below
      plan[0] = 0;
      plan[1] = 0;
    }
    mbar_init(bar(C_DRAIN), 1);
    mbar_init(bar(C_XCHG), 128);
    mbar_init(bar(C_O_READ), 128);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Rows qrows * g .. 127 of both Q tiles are never written by the Q loads: zero them once
  // (generic-proxy stores, made visible to the tensor cores' async proxy).
  {
    const int pad_chunks = (BM - qrows * a.group) * 16;
    for (int i = threadIdx.x; i < 2 * pad_chunks; i += kThreads2) {
      const int tile = i / pad_chunks, rem = i % pad_chunks;
      *reinterpret_cast<uint4*>(smem + Q2_OFF + tile * kTileBytes + sw_chunk(qrows * a.group + rem / 16, rem % 16)) =
          make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async();
  }
  // longest sequences first: order[rank] = b, ties by index
  if (sorted) {
    for (int b = threadIdx.x; b < a.batch; b += kThreads2) keys[b] = n_tiles_all - first_tile(b);
    __syncthreads();
    for (int b = threadIdx.x; b < a.batch; b += kThreads2) {
      const int k = keys[b];
      int rank = 0;
      for (int o = 0; o < a.batch; ++o) rank += (keys[o] > k) || (keys[o] == k && o < b);
      order[rank] = b;
      if (CHUNKS) {
        atomicAdd(plan, k);
        atomicMax(plan + 1, k);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // CHUNKS: when a sequence has more key tiles than a CTA's average share of the launch (tile
  // sum x items per sequence / grid), its items are split into key-range chunks of about that
  // share. Every CTA derives the same plan from the same keys.
  int split_avg = 0;
  bool chunks = false;
  if (CHUNKS && sorted) {
    split_avg = (int)(((long long)plan[0] * per_b + gridDim.x - 1) / gridDim.x);
    if (split_avg >= 1 && plan[1] > split_avg && (long long)a.batch * a.kv_heads * mtiles <= kPartCounters) {
      if (threadIdx.x == 0) {
        int n = 0, parts = 0;
        for (int r = 0; r < a.batch; ++r) {
          const int b = order[r];
          int len, nch;
          split_of(keys[b], split_avg, len, nch);
          start[r] = n;
          pbase[b] = parts;
          cinfo[b] = len | (nch << 16);
          n += per_b * nch;
          if (nch > 1) parts += a.kv_heads * mtiles * nch;
        }
        start[a.batch] = n;
        start[a.batch + 1] = parts <= kPartTiles ? 1 : 0;
      }
      __syncthreads();
      chunks = start[a.batch + 1] != 0;
      if (chunks) n_items = start[a.batch];
    }
  }
  const uint32_t tmem = *tmem_slot;
  // first key tile of sequence b, from the sort keys in shared memory when they exist
  auto tile0_of = [&](int b) { return sorted ? n_tiles_all - keys[b] : first_tile(b); };
  const int G = gridDim.x, c = blockIdx.x;
  // slot k of this CTA -> global position (snake order over the sorted list)
  auto item_at = [&](int k, Item& it) -> bool {
    const int p = k * G + ((k & 1) ? (G - 1 - c) : c);
    if (p >= n_items) return false;
    if (!CHUNKS || !chunks) {
      const int rank = p / per_b, rem = p % per_b;
      it.b = sorted ? order[rank] : rank;
      it.kvh = rem / pairs;
      it.pair = rem % pairs;
      return true;
    }
    int lo = 0, hi = a.batch;  // start[lo] <= p < start[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (start[mid] <= p) lo = mid;
      else hi = mid;
    }
    it.b = order[lo];
    int rem = p - start[lo];
    const int nch = cinfo[it.b] >> 16;
    const int chunk = rem % nch;
    rem /= nch;
    it.kvh = rem / pairs;
    it.pair = (rem % pairs) | (chunk << 16);
    return true;
  };
  // row-tile pair of an item, and its key tiles [lo, hi)
  auto pair_of = [&](const Item& x) { return CHUNKS ? (x.pair & 0xffff) : x.pair; };
  auto range_of = [&](const Item& x, int& lo, int& hi) {
    lo = tile0_of(x.b);
    hi = n_tiles_all;
    if (CHUNKS && chunks) {
      const int len = cinfo[x.b] & 0xffff;
      lo += (x.pair >> 16) * len;
      hi = min(hi, lo + len);
    }
  };

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
  if (warp == 0 || warp == 2 || warp == 3) {
    // ---------------- TMA producers ----------------
    // One thread issues TMA loads at about 50 GB/s (measured), below what an item start
    // needs (two Q tiles and the first K and V tiles at once), so three warps share the
    // work: warp 3 loads the Q tiles, warp 0 the K ring (and prefetches the next item into
    // L2), warp 2 the V ring. All walk the same item list.
    if (lane == 0) {
      const bool kq = warp == 0, qw = warp == 3;
      const CUtensorMap* map = qw ? &tmq : kq ? &tmk : &tmv;
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
      const int full0 = kq ? C_K_FULL : C_V_FULL, empty0 = kq ? C_K_EMPTY : C_V_EMPTY;
      const uint32_t ring = sbase + (kq ? K2_OFF : V2_OFF);
      // APPEND: the new rows' map and the pool map the tree tile is stored through
      const CUtensorMap* map_new = kq ? &am.k_new : &am.v_new;
      const CUtensorMap* map_pool = kq ? &am.k_pool : &am.v_pool;
      if (APPEND && !qw) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map_new)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map_pool)) : "memory");
      }
      int pend = -1, pend_cnt = 0, pend_b = 0, pend_h = 0;  // a loaded tree tile whose store is not issued
      bool reading[2] = {false, false};                     // a store may still read ring stage s
      // The tree tile of load `pend_cnt` has landed (its full barrier, which the MMA warp
      // also waits on): store it into the pools at position past. Issued one load later, so
      // the producer does not stall on the load it has just sent.
      auto store_tree = [&]() -> bool {
        if (!mbar_wait(bar(full0 + pend), (pend_cnt >> 1) & 1, abort_flag, a.err, kq ? 33 : 34)) return false;
        const uint32_t src = ring + pend * kTileBytes;
        tma_store_4d(map_pool, src, 0, a.past, pend_h, pend_b);
        tma_store_4d(map_pool, src + kTileHalf, 64, a.past, pend_h, pend_b);
        bulk_commit();
        reading[pend] = true;
        pend = -1;
        return true;
      };
      int cnt = 0, issued = 0;
      int qc[2] = {0, 0};                 // Q tiles requested per row tile
      bool q_issued[2] = {false, false};  // the latest request was sent (not withheld)
      const bool withhold = qw && blockIdx.x == 0 && *reinterpret_cast<volatile int*>(&g_withhold_q_arrival) != 0;
      const uint32_t q_bytes = 2u * 128u * (uint32_t)(qrows * a.group);  // two 64-dim halves of q * g rows
      bool ok = true;
      Item it;
      // K/V row of a sequence: through the row table when there is one
      auto kv_row = [&](int b, bool report) {
        if (!TABLE) return b;
        const long long p = kvr.map[b];
        if (p < 0 || p >= kvr.rows) {
          if (report) record_error(a.err, SPECKV_DERR_ROW_TABLE, p);
          return 0;
        }
        return (int)p;
      };
      for (int k = 0; ok && item_at(k, it); ++k) {
        // Q tiles of the item: each buffer is free once the previous item's last S MMA has read it
        const int ntq = !qw ? 0 : ((SPLIT || pair_of(it) * 2 + 1 >= mtiles) ? 1 : 2);
        for (int t = 0; t < ntq; ++t) {
          if (qc[t] >= 1 && !mbar_wait(bar(C_Q_EMPTY + t), (qc[t] - 1) & 1, abort_flag, a.err, 20)) { ok = false; break; }
          ++qc[t];
          q_issued[t] = !(withhold && k == 0 && t == 0);  // test hook: this tile never arrives
          if (!q_issued[t]) continue;
          const uint32_t qd = sbase + Q2_OFF + t * kTileBytes;
          const int r0 = SPLIT ? 0 : (pair_of(it) * 2 + t) * qrows;
          mbar_expect_tx(bar(C_Q_FULL + t), q_bytes);
          tma_load_4d(qd, &tmq, bar(C_Q_FULL + t), 0, it.kvh * a.group, r0, it.b);
          tma_load_4d(qd + kTileHalf, &tmq, bar(C_Q_FULL + t), 64, it.kvh * a.group, r0, it.b);
        }
        if (!ok) break;
        if (qw) continue;  // warp 3 loads only the Q tiles
        int t0, t1;
        range_of(it, t0, t1);
        const int kb = kv_row(it.b, kq);
        // three key tiles before this item ends, the next item's Q tiles and first K / V
        // tiles are prefetched into L2, so that its start does not wait on DRAM
        const int prefetch_at = max(t0, t1 - 3);
        for (int i = t0; i < t1; ++i, ++cnt) {
          const int s = cnt & 1;
          Item nx;
          if (kq && i == prefetch_at && item_at(k + 1, nx)) {
            const int nq = (SPLIT || pair_of(nx) * 2 + 1 >= mtiles) ? 1 : 2;
            for (int t = 0; t < nq; ++t)
              for (int h = 0; h < 2; ++h)
                tma_prefetch_4d(&tmq, h * 64, nx.kvh * a.group, SPLIT ? 0 : (pair_of(nx) * 2 + t) * qrows, nx.b);
            int nt0, nt1;
            range_of(nx, nt0, nt1);
            const int nkb = kv_row(nx.b, false);
            for (int j = nt0; j < nt0 + 2 && j < nt1; ++j)
              for (int h = 0; h < 2; ++h) {
                if (APPEND && j == n_cached) {
                  tma_prefetch_4d(&am.k_new, h * 64, 0, nx.kvh, nx.b);
                  tma_prefetch_4d(&am.v_new, h * 64, 0, nx.kvh, nx.b);
                } else {
                  tma_prefetch_4d(&tmk, h * 64, j * BN, nx.kvh, nkb);
                  tma_prefetch_4d(&tmv, h * 64, j * BN, nx.kvh, nkb);
                }
              }
          }
          if (APPEND && pend >= 0 && !store_tree()) {
            ok = false;
            break;
          }
          if (cnt >= 2 && !mbar_wait(bar(empty0 + s), ((cnt >> 1) - 1) & 1, abort_flag, a.err, kq ? 21 : 22)) {
            ok = false;
            break;
          }
          if (APPEND && reading[s]) {  // a tree-tile store still reads this stage
            bulk_wait_read_all();
            reading[0] = reading[1] = false;
          }
          const uint32_t dst = ring + s * kTileBytes;
          mbar_expect_tx(bar(full0 + s), kTileBytes);
          if (APPEND && i == n_cached) {
            tma_load_4d(dst, map_new, bar(full0 + s), 0, 0, it.kvh, it.b);
            tma_load_4d(dst + kTileHalf, map_new, bar(full0 + s), 64, 0, it.kvh, it.b);
            if (pair_of(it) == 0) {  // one item per (sequence, KV head) appends its rows
              pend = s;
              pend_cnt = cnt;
              pend_b = it.b;
              pend_h = it.kvh;
            }
          } else {
            tma_load_4d(dst, map, bar(full0 + s), 0, i * BN, it.kvh, kb);
            tma_load_4d(dst + kTileHalf, map, bar(full0 + s), 64, i * BN, it.kvh, kb);
          }
          issued = cnt + 1;
        }
      }
      if (APPEND) {
        if (ok && pend >= 0) store_tree();
        bulk_wait_all();  // every store has completed before the CTA exits
      }
      // Loads still in flight must land before shared memory is released: after an abort
      // (which may come after this loop ended) nobody consumes them; in a normal run
      // these phases completed long ago and the waits return at once.
      for (int q = issued - 2 < 0 ? 0 : issued - 2; q < issued; ++q) drain_wait(bar(full0 + (q & 1)), (q >> 1) & 1);
      for (int t = 0; t < 2; ++t)
        if (qc[t] >= 1 && q_issued[t]) drain_wait(bar(C_Q_FULL + t), (qc[t] - 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp, lane 0 issues) ----------------
    {
      const uint32_t ab = TypeCode<T>::value;
      const uint32_t id_s = idesc_f16(ab, 0), id_pv = idesc_f16(ab, 1);
      int cnt = 0;            // key tiles consumed (global)
      int sc[2] = {0, 0};     // S / P completions per row tile
      int ic[2] = {0, 0};     // items per row tile
      bool ok = true;
      Item it;
      auto wait = [&](int b, uint32_t parity, int where) {
        return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, abort_flag, a.err, where));
      };
      // Descriptor bases, computed once; a K step only adds a constant to the
      // start-address field (16-byte units): K-major +32 B per 16 elements inside a
      // 128-byte swizzle atom and +16 KB per 64-element half, V (MN-major) +2 KB; a
      // ring stage adds kTileBytes.
      const uint64_t q_desc = sw128_desc(sbase + Q2_OFF, 16, 1024);
      const uint64_t k_desc = sw128_desc(sbase + K2_OFF, 16, 1024);
      const uint64_t v_desc = sw128_desc(sbase + V2_OFF, kTileHalf, 1024);
      constexpr uint64_t kStageStep = kTileBytes >> 4;
      // descriptors are computed by the whole warp (warp-uniform); one elected lane issues
      // the group of MMAs and its commit
      auto issue_s = [&](int t, int stage, int qt) {
        const uint64_t ad = q_desc + (uint64_t)qt * kStageStep, bd = k_desc + (uint64_t)stage * kStageStep;
        const uint32_t d = tmem + S_COL(t);
        const uint32_t sbar = bar(C_S_FULL + t);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t step = (uint64_t)((kk >> 2) * (kTileHalf >> 4) + (kk & 3) * 2);
            tc_mma(d, ad + step, bd + step, id_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(sbar);
        }
        __syncwarp();
      };
      // P.V in two halves: keys 0..63 as soon as the softmax has stored that half of P
      // (C_PH_FULL), keys 64..127 after the rest (C_P_FULL). SPLIT publishes P at once and
      // issues all eight MMAs after C_P_FULL (fewer live registers in its MMA warp).
      auto issue_pv = [&](int t, int stage, bool first) -> bool {
        const uint64_t bd = v_desc + (uint64_t)stage * kStageStep;
        const uint32_t d = tmem + O2_COL(t), pa = tmem + S_COL(t);
        const uint32_t acc0 = first ? 0u : 1u;
        if (!SPLIT) {
          if (!wait(C_PH_FULL + t, sc[t] & 1, 32)) return false;
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < BN / 32; ++kk)
              tc_mma_ts(d, pa + kk * 8, bd + (uint64_t)(kk * (2048 >> 4)), id_pv, kk > 0 ? 1u : acc0);
          }
          __syncwarp();
        }
        if (!wait(C_P_FULL + t, sc[t] & 1, 23)) return false;
        ++sc[t];
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int kk = SPLIT ? 0 : BN / 32; kk < BN / 16; ++kk)
            tc_mma_ts(d, pa + kk * 8, bd + (uint64_t)(kk * (2048 >> 4)), id_pv, kk > 0 ? 1u : acc0);
        }
        __syncwarp();
        return true;
      };
      for (int k = 0; ok && item_at(k, it); ++k) {
        if (SPLIT) {
          int r0, r1;
          range_of(it, r0, r1);
          const int n = r1 - r0;
          ok = wait(C_Q_FULL + 0, ic[0] & 1, 24);
          tc_fence_after();
          // O0 and O1 of the previous item must be read (merged) before this item's first P.V
          bool o_busy = ic[0] >= 1;
          auto o_free = [&]() -> bool {
            if (!o_busy) return true;
            o_busy = false;
            if (!wait(C_O_READ, (ic[0] - 1) & 1, 31)) return false;
            tc_fence_after();
            return true;
          };
          int prev_stage = 0;
          for (int i = 0; ok && i < n; ++i, ++cnt) {
            const int s = cnt & 1, w = i & 1;
            if (!wait(C_K_FULL + s, (cnt >> 1) & 1, 26)) { ok = false; break; }
            tc_fence_after();
            issue_s(w, s, 0);
            tc_commit_w(bar(C_K_EMPTY + s));
            if (i == n - 1) tc_commit_w(bar(C_Q_EMPTY + 0));  // the last S MMA has read Q
            if (i > 0) {  // P.V of the previous tile, the other warpgroup's
              if (!wait(C_V_FULL + prev_stage, ((cnt - 1) >> 1) & 1, 27)) { ok = false; break; }
              tc_fence_after();
              if (!o_free() || !issue_pv(1 - w, prev_stage, i - 1 < 2)) { ok = false; break; }
              tc_commit_w(bar(C_V_EMPTY + prev_stage));
            }
            prev_stage = s;
          }
          if (ok && n > 0) {
            if (!wait(C_V_FULL + prev_stage, ((cnt - 1) >> 1) & 1, 27)) {
              ok = false;
            } else {
              tc_fence_after();
              if (o_free() && issue_pv((n - 1) & 1, prev_stage, n - 1 < 2)) tc_commit_w(bar(C_V_EMPTY + prev_stage));
              else ok = false;
            }
          }
          if (!ok) break;
          tc_commit_w(bar(C_O_FINAL + 0));
          tc_commit_w(bar(C_O_FINAL + 1));
          ++ic[0];
          ++ic[1];
          continue;
        }
        const bool act1 = pair_of(it) * 2 + 1 < mtiles;
        int r0, r1;
        range_of(it, r0, r1);
        const int n = r1 - r0;
        ok = wait(C_Q_FULL + 0, ic[0] & 1, 24);
        if (ok && act1) ok = wait(C_Q_FULL + 1, ic[1] & 1, 25);
        tc_fence_after();
        int prev_stage = 0;
        for (int i = 0; ok && i < n; ++i, ++cnt) {
          const int s = cnt & 1;
          if (!wait(C_K_FULL + s, (cnt >> 1) & 1, 26)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, s, 0);
          if (act1 && i > 0) {
            if (!issue_pv(1, prev_stage, i == 1)) { ok = false; break; }
            tc_commit_w(bar(C_V_EMPTY + prev_stage));
          }
          if (act1) issue_s(1, s, 1);
          tc_commit_w(bar(C_K_EMPTY + s));
          if (i == n - 1) {  // the last S MMAs have read the Q tiles: the next item's Q may load
            tc_commit_w(bar(C_Q_EMPTY + 0));
            if (act1) tc_commit_w(bar(C_Q_EMPTY + 1));
          }
          if (!wait(C_V_FULL + s, (cnt >> 1) & 1, 27)) { ok = false; break; }
          tc_fence_after();
          if (!issue_pv(0, s, i == 0)) { ok = false; break; }
          if (!act1) tc_commit_w(bar(C_V_EMPTY + s));
          if (i == n - 1) tc_commit_w(bar(C_O_FINAL + 0));  // O0 is final: its epilogue need not wait for P1
          prev_stage = s;
        }
        if (ok && act1) {
          if (issue_pv(1, prev_stage, n == 1)) tc_commit_w(bar(C_V_EMPTY + prev_stage));
          else ok = false;
        }
        if (!ok) break;
        ++ic[0];
        if (act1) {
          tc_commit_w(bar(C_O_FINAL + 1));
          ++ic[1];
        }
      }
      tc_commit_w(bar(C_DRAIN));  // every MMA of lane 0 completes before TMEM is released
      drain_wait(bar(C_DRAIN), 0);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ---------------- softmax warpgroups ----------------
    const int t = (warp - 4) >> 2;                 // row tile of this warpgroup
    const int quarter = warp & 3;                  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;           // row within the tile == TMEM lane
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + S_COL(t);
    const uint32_t o_addr = tmem + lane_addr + O2_COL(t);
    const float scale = a.scale_log2;
    struct RowMap {
      bool valid;
      int r, hq;
    };
    // tile row -> (tree row, query head): the packing of the Q tensor map's boxes
    auto row_map = [&](const Item& x) {
      RowMap m;
      const int tile = SPLIT ? 0 : pair_of(x) * 2 + t;
      const int rr = tile * qrows + row / a.group;
      m.valid = row < qrows * a.group && rr < a.rows;
      m.r = m.valid ? rr : 0;
      m.hq = x.kvh * a.group + (m.valid ? row % a.group : 0);
      return m;
    };
    auto next_item = [&](int& kk, Item& nx) -> bool {
      for (;; ++kk) {
        if (!item_at(kk, nx)) return false;
        if (SPLIT || t == 0 || pair_of(nx) * 2 + 1 < mtiles) return true;
      }
    };
    const bool out32 = (reinterpret_cast<uintptr_t>(a.out) & 31u) == 0;  // 32-byte output stores
    int sc = 0, ic = 0, k = 0;
    bool ok = true;
    Item it;
    bool have = next_item(k, it);
    const int i_first = SPLIT ? t : 0, i_step = SPLIT ? 2 : 1;  // this warpgroup's key tiles
    while (have) {
      int t0, t1;
      range_of(it, t0, t1);
      const int n = t1 - t0;
      const RowMap m = row_map(it);
      const uint32_t* brow = a.bits + ((long long)it.b * a.rows + m.r) * a.row_words + t0 * 4;
      float m_run = -INFINITY, l_run = 0.f;
      for (int i = i_first; i < n; i += i_step) {
        uint4 w = make_uint4(0, 0, 0, 0);
        if (!APPEND) {
          if (m.valid) w = *reinterpret_cast<const uint4*>(brow + i * 4);
        } else if (m.valid) {
          // cached tile: its words, cut at past; tree tile: the words from bit past on, cut at
          // the row count (the words are read one by one inside the row)
          const int g = t0 + i;
          int lim;
          if (g < n_cached) {
            w = *reinterpret_cast<const uint4*>(brow + i * 4);
            lim = a.past - g * BN;
          } else {
            const uint32_t* rw = brow - t0 * 4;
            const int wq = a.past >> 5, sh = a.past & 31;
            uint32_t u[5];
#pragma unroll
            for (int q = 0; q < 5; ++q) u[q] = wq + q < a.row_words ? rw[wq + q] : 0u;
            w = make_uint4(__funnelshift_r(u[0], u[1], sh), __funnelshift_r(u[1], u[2], sh),
                           __funnelshift_r(u[2], u[3], sh), __funnelshift_r(u[3], u[4], sh));
            lim = a.rows;
          }
          if (lim < BN) {
            w.x &= low_bits(lim);
            w.y &= low_bits(lim - 32);
            w.z &= low_bits(lim - 64);
            w.w &= low_bits(lim - 96);
          }
        }
        ok = mbar_wait(bar(C_S_FULL + t), sc & 1, abort_flag, a.err, 28);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        float x[BN];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) tmem_ld32(s_addr + cc * 32, x + cc * 32);
        tmem_wait_ld();
        const bool dense = __all_sync(0xffffffffu, (w.x & w.y & w.z & w.w) == 0xffffffffu);
        if (!dense) {
          const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < BN; ++j) x[j] = ((words[j >> 5] >> (j & 31)) & 1u) ? x[j] : -INFINITY;
        }
        float mx0 = fmax3(x[0], x[1], x[2]), mx1 = fmax3(x[3], x[4], x[5]);
#pragma unroll
        for (int j = 6; j + 3 < BN; j += 4) {  // columns 6 .. 125
          mx0 = fmax3(mx0, x[j], x[j + 1]);
          mx1 = fmax3(mx1, x[j + 2], x[j + 3]);
        }
        const float mxs = fmax3(mx0, mx1, fmaxf(x[BN - 2], x[BN - 1])) * scale;
        const bool grow_max = mxs > m_run + 8.0f;
        const float m_new = grow_max ? mxs : m_run;
        const float corr = (grow_max && m_run != -INFINITY) ? ex2(m_run - m_new) : 1.f;
        m_run = m_new;
        const float2 sc2 = make_float2(scale, scale);
        const float nm = m_run == -INFINITY ? 0.f : -m_run;
        const float2 neg = make_float2(nm, nm);
        float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};  // independent partial sums: no 64-long add chain
        // P = 2^(s * scale - m), packed to 16 bits over the first 64 columns of S, in two
        // halves of 64 keys (the first half's P.V starts while the second is computed);
        // pairs on the MUFU ex2 unit or by polynomial on the FMA pipe (poly_pair)
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t pk[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            float2 e = __ffma2_rn(make_float2(x[cc * 16 + j], x[cc * 16 + j + 1]), sc2, neg);
            if (poly_pair(j >> 1)) {
              e = exp2_poly2(e);
            } else {
              e.x = ex2(e.x);
              e.y = ex2(e.y);
            }
            sum2[(j >> 1) & 3] = __fadd2_rn(sum2[(j >> 1) & 3], e);
            pk[j >> 1] = pack2<T>(e.x, e.y);
          }
          tmem_st8(s_addr + cc * 8, pk);
          // O is rescaled before the first P.V of this tile: after the first half of P (only
          // 64 scores still live) when the halves are published apart, else after all of P
          if (cc == (SPLIT ? 7 : 3)) {
            if (i > i_first && __any_sync(0xffffffffu, corr != 1.f)) {
              // O_t holds tiles < i: their P.V MMAs were issued before S_t,i, and the commit
              // that signalled S_t,i covers them; P_t,i . V_i waits for C_PH_FULL below.
#pragma unroll
              for (int oc = 0; oc < 4; ++oc) {
                float o[32];
                tmem_ld32(o_addr + oc * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] *= corr;
                tmem_st32(o_addr + oc * 32, o);
              }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C_PH_FULL + t));
          }
        }
        // (SPLIT: the draft-sized kernel publishes both halves at once, which keeps its
        // register footprint)
        if (!SPLIT) {
          tmem_wait_st();
          tc_fence_before();
        }
        mbar_arrive(bar(C_P_FULL + t));
        const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
        l_run = l_run * corr + ((s01.x + s01.y) + (s23.x + s23.y));
      }
      if (!ok) break;
      Item nx;
      int kn = k + 1;
      const bool have_next = next_item(kn, nx);
      ok = mbar_wait(bar(C_O_FINAL + t), ic & 1, abort_flag, a.err, 29);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      if (CHUNKS && !SPLIT && chunks && (cinfo[it.b] >> 16) > 1) {
        // one chunk of a split row tile: its unnormalised O, running max and sum go to the
        // launch's partials; the warpgroup that completes the tile's last chunk merges
        ++ic;
        const int nch = cinfo[it.b] >> 16;
        const int tile = pair_of(it) * 2 + t, chunk = it.pair >> 16;
        float* const parts = g_part + ((size_t)a.part_slot * kPartTiles + pbase[it.b] +
                                       (it.kvh * mtiles + tile) * nch) * kPartTileFloats;
        float* const prow = parts + (size_t)chunk * kPartTileFloats + row * kPartRowFloats;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float o[32];
          tmem_ld32(o_addr + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(reinterpret_cast<float4*>(prow + cc * 32 + j), make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]));
        }
        __stcg(reinterpret_cast<float2*>(prow + 128), make_float2(m_run, l_run));
        tc_fence_before();
        __threadfence();
        asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");
        int* const counter = g_part_count + (size_t)a.part_slot * kPartCounters +
                             ((long long)it.b * a.kv_heads + it.kvh) * mtiles + tile;
        if (row == 0) lastf[t] = atomicAdd(counter, 1) == nch - 1 ? 1 : 0;
        asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");
        if (lastf[t]) {
          __threadfence();
          const float* const rows0 = parts + row * kPartRowFloats;
          float mm = -INFINITY;
          for (int cc = 0; cc < nch; ++cc) mm = fmaxf(mm, __ldcg(rows0 + (size_t)cc * kPartTileFloats + 128));
          float l = 0.f;
          for (int cc = 0; cc < nch; ++cc) {
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(rows0 + (size_t)cc * kPartTileFloats + 128));
            l += ml.x == -INFINITY ? 0.f : ml.y * ex2(ml.x - mm);
          }
          const float inv_l = l > 0.f ? 1.f / l : 0.f;
          T* orow = static_cast<T*>(a.out) + (((long long)it.b * a.rows + m.r) * a.q_heads + m.hq) * HD;
#pragma unroll 1
          for (int cb = 0; cb < 4; ++cb) {
            float acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.f;
            for (int cc = 0; cc < nch; ++cc) {
              const float* src = rows0 + (size_t)cc * kPartTileFloats;
              const float mc = __ldcg(src + 128);
              const float w = mc == -INFINITY ? 0.f : ex2(mc - mm) * inv_l;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(src + cb * 32 + j));
                acc[j] += w * v.x;
                acc[j + 1] += w * v.y;
                acc[j + 2] += w * v.z;
                acc[j + 3] += w * v.w;
              }
            }
            if (m.valid) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 v;
                v.x = pack2<T>(acc[j], acc[j + 1]);
                v.y = pack2<T>(acc[j + 2], acc[j + 3]);
                v.z = pack2<T>(acc[j + 4], acc[j + 5]);
                v.w = pack2<T>(acc[j + 6], acc[j + 7]);
                *reinterpret_cast<uint4*>(orow + cb * 32 + j) = v;
              }
            }
          }
          if (row == 0) atomicExch(counter, 0);  // ready for the slot's next launch
        }
        it = nx;
        k = kn;
        have = have_next;
        continue;
      }
      float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      float c0 = 1.f, c1 = 0.f;  // SPLIT: weights of O0 and O1 in the merged output
      bool use1 = false;
      if (SPLIT) {
        float2* xch = reinterpret_cast<float2*>(smem + Q2_OFF + kTileBytes);  // Q tile 1 is unused
        if (t == 1) {
          xch[row] = make_float2(m_run, l_run);
          mbar_arrive(bar(C_XCHG));
          ++ic;
          it = nx;
          k = kn;
          have = have_next;
          continue;
        }
        ok = mbar_wait(bar(C_XCHG), ic & 1, abort_flag, a.err, 30);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        const float2 ml1 = xch[row];
        const float mm = fmaxf(m_run, ml1.x);
        c0 = m_run == -INFINITY ? 0.f : ex2(m_run - mm);
        use1 = ml1.x != -INFINITY;
        c1 = use1 ? ex2(ml1.x - mm) : 0.f;
        const float l = l_run * c0 + (use1 ? ml1.y * c1 : 0.f);
        inv = l > 0.f ? 1.f / l : 0.f;
      }
      ++ic;
      T* orow = static_cast<T*>(a.out) + (((long long)it.b * a.rows + m.r) * a.q_heads + m.hq) * HD;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float o[64];
        tmem_ld32(o_addr + cc * 64, o);
        tmem_ld32(o_addr + cc * 64 + 32, o + 32);
        tmem_wait_ld();
        if (SPLIT) {
          const uint32_t o1_addr = tmem + lane_addr + O2_COL(1) + cc * 64;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float o1[32];
            tmem_ld32(o1_addr + h * 32, o1);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[h * 32 + j] = o[h * 32 + j] * c0 + (use1 ? o1[j] * c1 : 0.f);
          }
        }
        if (m.valid && out32) {  // whole 32-byte sectors: half the store transactions
#pragma unroll
          for (int j = 0; j < 64; j += 16) {
            uint32_t w[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w[e] = pack2<T>(o[j + 2 * e] * inv, o[j + 2 * e + 1] * inv);
            st_global_v8(orow + cc * 64 + j, w);
          }
        } else if (m.valid) {
#pragma unroll
          for (int j = 0; j < 64; j += 8) {
            uint4 v;
            v.x = pack2<T>(o[j] * inv, o[j + 1] * inv);
            v.y = pack2<T>(o[j + 2] * inv, o[j + 3] * inv);
            v.z = pack2<T>(o[j + 4] * inv, o[j + 5] * inv);
            v.w = pack2<T>(o[j + 6] * inv, o[j + 7] * inv);
            *reinterpret_cast<uint4*>(orow + cc * 64 + j) = v;
          }
        }
      }
      tc_fence_before();
      if (SPLIT) mbar_arrive(bar(C_O_READ));  // O0 and O1 are read: the next item's P.V may start
      it = nx;
      k = kn;
      have = have_next;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Encoded maps of the views seen last on this thread: the verify loop hands every layer's
// K/V cache views and query projections again each round, so their maps are encoded once.
struct MapEntry {
  const void* base;
  long long dims[3], strides[3];
  int box1, box2, dtype;
  CUtensorMap map;
};
constexpr int kMapCache = 512;

// 4-D map with a 128-element (head dim) innermost dimension, 128-byte swizzle and a box of
// (64, box1, box2, 1): dims[i] / strides[i] (elements) are the three outer dimensions.
bool make_map(CUtensorMap* map, const void* base, const long long* dims, const long long* strides, int box1,
              int box2, int dtype) {
  thread_local MapEntry cache[kMapCache];
  thread_local int used = 0, next = 0;
  for (int i = 0; i < used; ++i) {
    const MapEntry& e = cache[i];
    if (e.base == base && e.dims[0] == dims[0] && e.dims[1] == dims[1] && e.dims[2] == dims[2] &&
        e.strides[0] == strides[0] && e.strides[1] == strides[1] && e.strides[2] == strides[2] &&
        e.box1 == box1 && e.box2 == box2 && e.dtype == dtype) {
      *map = e.map;
      return true;
    }
  }
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t gdims[4] = {(cuuint64_t)HD, (cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2]};
  const cuuint64_t gstrides[3] = {(cuuint64_t)strides[0] * 2, (cuuint64_t)strides[1] * 2,
                                  (cuuint64_t)strides[2] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box1, (cuuint32_t)box2, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult res = fn(map, dtype == SPECKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    4, const_cast<void*>(base), gdims, gstrides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return false;
  MapEntry& e = cache[next];
  e.base = base;
  for (int i = 0; i < 3; ++i) {
    e.dims[i] = dims[i];
    e.strides[i] = strides[i];
  }
  e.box1 = box1;
  e.box2 = box2;
  e.dtype = dtype;
  e.map = *map;
  next = (next + 1) % kMapCache;
  if (used < kMapCache) ++used;
  return true;
}

// K or V: a (batch, heads, len, 128) strided view -> dims (d, len, heads, batch), box of
// 64 dims x BN positions.
bool make_kv_map(CUtensorMap* map, const void* base, const long long* st, long long batch, long long heads,
                 long long len, int dtype) {
  const long long dims[3] = {len, heads, batch}, strides[3] = {st[2], st[1], st[0]};
  return make_map(map, base, dims, strides, BN, 1, dtype);
}

// Q: a (batch, q_heads, rows, 128) strided view -> dims (d, q_heads, rows, batch), box of
// 64 dims x g heads x floor(128 / g) tree rows (one row tile of the pair kernel).
bool make_q_map(CUtensorMap* map, const void* base, const long long* st, long long batch, long long q_heads,
                long long rows, int group, int dtype) {
  const long long dims[3] = {q_heads, rows, batch}, strides[3] = {st[1], st[2], st[0]};
  return make_map(map, base, dims, strides, group, BM / group, dtype);
}

template <typename T, int MODE, typename MT>
int launch_sm100(const CUtensorMap& mk, const CUtensorMap& mv, const Sm100Args& s, cudaStream_t stream) {
  auto kern = attn_sm100_kernel<T, MODE, MT>;
  const uint32_t smem = SMEM_BYTES + (MODE == 2 ? 2 * mask_stage_bytes<MT>() : 0u);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const long long grid = (long long)s.batch * s.kv_heads * s.mtiles;
  kern<<<(unsigned)grid, kThreads, smem, stream>>>(mk, mv, s);
  return check_launch("speckv_tree_attention(sm100)");
}

constexpr int kMaxAttnDevices = 64;

int current_device() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxAttnDevices ? dev : -1;
}

// Upper bound on the persistent attention grid (0: one CTA per SM). A job whose collectives run
// beside the attention (a counter all_reduce on a side stream) leaves their SMs free with it.
int g_attention_ctas = 0;

// Key-range chunks for long sequences (speckv_attention_set_chunks): off by default.
int g_attention_chunks = 0;

int sm_count() {
  static int cached[kMaxAttnDevices] = {0};
  const int dev = current_device();
  if (dev >= 0 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  cached[dev] = n;
  return n;
}

template <typename T, bool SPLIT, bool TABLE, bool CHUNKS = false, bool APPEND = false>
int launch_pair(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, const Sm100Args& s,
                const KvRows& kvr, cudaStream_t stream, const AppendMaps* am = nullptr) {
  auto kern = attn_pair_kernel<T, SPLIT, TABLE, CHUNKS, APPEND>;
  constexpr uint32_t smem_bytes = CHUNKS ? SMEM2C_BYTES : SMEM2_BYTES;
  // The setmaxnreg split assumes the block starts with exactly kRegsLaunch registers
  // per thread; any other count could leave the increase waiting for registers.
  static int regs = -1;
  if (regs < 0) {
    cudaFuncAttributes fa;
    regs = cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : 0;
  }
  if (regs != kRegsLaunch)
    return fail(SPECKV_ENOSUPPORT, "speckv_tree_attention_bits: kernel compiled with %d registers per thread, "
                "the register split needs %d", regs, kRegsLaunch);
  static bool smem_set[kMaxAttnDevices] = {false};  // the attribute is per device: set it once on each
  const int dev = current_device();
  if (dev < 0 || !smem_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
    if (dev >= 0) smem_set[dev] = true;
  }
  const long long qrows = BM / s.group, mtiles = (s.rows + qrows - 1) / qrows;
  const long long pairs = SPLIT ? 1 : (mtiles + 1) / 2;
  const long long items = (long long)s.batch * s.kv_heads * pairs;
  long long ctas = sm_count();
  if (g_attention_ctas > 0 && g_attention_ctas < ctas) ctas = g_attention_ctas;
  // with key-range chunks a launch can have more items than this count: a full grid then
  const long long grid = CHUNKS ? ctas : (items < ctas ? items : ctas);
  Sm100Args sa = s;
  if (CHUNKS) {
    static bool parts_zeroed[kMaxAttnDevices] = {false};  // the merge counters start at zero
    if (dev >= 0 && !parts_zeroed[dev]) {
      if (attention_reset_partials() != SPECKV_OK) return SPECKV_ECUDA;
      parts_zeroed[dev] = true;
    }
    // launches that may run at the same time (on other streams) take different slots
    static std::atomic<unsigned> next_slot{0};
    sa.part_slot = (int)(next_slot.fetch_add(1u) % (unsigned)kPartSlots);
  }
  static const AppendMaps no_append{};  // the argument of the instantiations without the append
  kern<<<(unsigned)grid, kThreads2, smem_bytes, stream>>>(mk, mv, mq, sa, kvr, am != nullptr ? *am : no_append);
  return check_launch(APPEND ? "speckv_tree_attention_bits_append(sm100)" : "speckv_tree_attention_bits(sm100)");
}

}  // namespace

void attention_set_ctas(int ctas) { g_attention_ctas = ctas > 0 ? ctas : 0; }

void attention_set_chunks(int on) { g_attention_chunks = on ? 1 : 0; }

int attention_test_hooks(long long wait_limit_ns, int withhold_q_arrival) {
  const unsigned long long lim = wait_limit_ns > 0 ? (unsigned long long)wait_limit_ns : 0ull;
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &lim, sizeof(lim));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_withhold_q_arrival, &withhold_q_arrival, sizeof(int));
  if (e != cudaSuccess) return fail(SPECKV_ECUDA, "speckv_attention_test_hooks: %s", cudaGetErrorString(e));
  return attention_reset_partials();
}

int attention_reset_partials() {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_part_count);
  if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(g_part_count));
  if (e != cudaSuccess) return fail(SPECKV_ECUDA, "attention partials reset: %s", cudaGetErrorString(e));
  return SPECKV_OK;
}

bool sm100_supported(const AttnArgs& a) {
  if (a.dim != HD || (a.dtype != SPECKV_BF16 && a.dtype != SPECKV_F16)) return false;
  const long long* strides[3] = {a.qs, a.ks, a.vs};
  for (const long long* st : strides)
    for (int i = 0; i < 3; ++i)
      if ((st[i] * 2) % 16 != 0) return false;
  if (((uintptr_t)a.q | (uintptr_t)a.k | (uintptr_t)a.v | (uintptr_t)a.out) % 16 != 0) return false;
  if (a.batch > (1 << 20) || a.kv_len > (1 << 30)) return false;
  // visibility words are read 16 bytes at a time
  if (a.bits != nullptr && (a.row_words % 4 != 0 || (uintptr_t)a.bits % 16 != 0)) return false;
  if (a.past >= 0) {  // the appended rows are read by TMA as well
    for (int i = 0; i < 3; ++i)
      if ((a.kns[i] * 2) % 16 != 0 || (a.vns[i] * 2) % 16 != 0) return false;
    if (((uintptr_t)a.k_new | (uintptr_t)a.v_new) % 16 != 0) return false;
  }
  return true;
}

int attention_sm100(const AttnArgs& a, cudaStream_t stream) {
  const uint32_t* bits = a.bits;
  const bool append = a.past >= 0;
  // with the append fused the pools are read over the cached positions only (an empty
  // cache still gets a valid one-position map, which no tile reads)
  const long long load_len = append ? (a.past > 0 ? a.past : 1) : a.kv_len;
  CUtensorMap mk, mv;
  if (!make_kv_map(&mk, a.k, a.ks, a.kv_batch, a.kv_heads, load_len, a.dtype) ||
      !make_kv_map(&mv, a.v, a.vs, a.kv_batch, a.kv_heads, load_len, a.dtype))
    return fail(SPECKV_ECUDA, "speckv_tree_attention: cuTensorMapEncodeTiled failed");
  unsigned long long* err = device_error_word();
  if (err == nullptr) return fail(SPECKV_ECUDA, "speckv_tree_attention: device error word unavailable");
  Sm100Args s;
  s.q = a.q;
  s.qs0 = a.qs[0];
  s.qs1 = a.qs[1];
  s.qs2 = a.qs[2];
  s.out = a.out;
  s.bits = bits;
  s.row_words = a.row_words;
  s.first_col = a.first_col;
  s.mask = a.mask;
  s.mask_dtype = a.mask_dtype;
  s.batch = (int)a.batch;
  s.q_heads = (int)a.q_heads;
  s.kv_heads = (int)a.kv_heads;
  s.group = (int)(a.q_heads / a.kv_heads);
  s.rows = (int)a.rows;
  s.kv_len = (int)a.kv_len;
  s.mtiles = (int)((s.group * a.rows + BM - 1) / BM);
  s.scale_log2 = a.scale * 1.4426950408889634f;
  s.part_slot = 0;
  s.past = append ? (int)a.past : 0;
  s.err = err;
  const KvRows kvr{a.row_table, (int)a.kv_batch};
  const bool bf = a.dtype == SPECKV_BF16;
  if (bits != nullptr) {
    if (s.group > BM)
      return fail(SPECKV_ENOSUPPORT, "speckv_tree_attention_bits: %d query heads per KV head (at most %d)", s.group,
                  BM);
    CUtensorMap mq;
    if (!make_q_map(&mq, a.q, a.qs, a.batch, a.q_heads, a.rows, s.group, a.dtype))
      return fail(SPECKV_ECUDA, "speckv_tree_attention_bits: cuTensorMapEncodeTiled failed for the query");
    // at most one 128-row tile per (sequence, KV head): the two warpgroups split the keys
    const bool split = (long long)s.group * s.rows <= BM, table = kvr.map != nullptr;
    if (append) {
      AppendMaps am;
      if (!make_kv_map(&am.k_new, a.k_new, a.kns, a.batch, a.kv_heads, a.rows, a.dtype) ||
          !make_kv_map(&am.v_new, a.v_new, a.vns, a.batch, a.kv_heads, a.rows, a.dtype) ||
          !make_kv_map(&am.k_pool, a.k, a.ks, a.kv_batch, a.kv_heads, a.past + a.rows, a.dtype) ||
          !make_kv_map(&am.v_pool, a.v, a.vs, a.kv_batch, a.kv_heads, a.past + a.rows, a.dtype))
        return fail(SPECKV_ECUDA, "speckv_tree_attention_bits_append: cuTensorMapEncodeTiled failed");
      if (bf) return split ? launch_pair<__nv_bfloat16, true, false, false, true>(mk, mv, mq, s, kvr, stream, &am)
                           : launch_pair<__nv_bfloat16, false, false, false, true>(mk, mv, mq, s, kvr, stream, &am);
      return split ? launch_pair<__half, true, false, false, true>(mk, mv, mq, s, kvr, stream, &am)
                   : launch_pair<__half, false, false, false, true>(mk, mv, mq, s, kvr, stream, &am);
    }
    if (bf) {
      if (split) return table ? launch_pair<__nv_bfloat16, true, true>(mk, mv, mq, s, kvr, stream)
                              : launch_pair<__nv_bfloat16, true, false>(mk, mv, mq, s, kvr, stream);
      if (g_attention_chunks && !table) return launch_pair<__nv_bfloat16, false, false, true>(mk, mv, mq, s, kvr, stream);
      return table ? launch_pair<__nv_bfloat16, false, true>(mk, mv, mq, s, kvr, stream)
                   : launch_pair<__nv_bfloat16, false, false>(mk, mv, mq, s, kvr, stream);
    }
    if (split) return table ? launch_pair<__half, true, true>(mk, mv, mq, s, kvr, stream)
                            : launch_pair<__half, true, false>(mk, mv, mq, s, kvr, stream);
    if (g_attention_chunks && !table) return launch_pair<__half, false, false, true>(mk, mv, mq, s, kvr, stream);
    return table ? launch_pair<__half, false, true>(mk, mv, mq, s, kvr, stream)
                 : launch_pair<__half, false, false>(mk, mv, mq, s, kvr, stream);
  }
  const int min_group = a.mask_dtype == SPECKV_F32 ? mask_min_group<float>() : mask_min_group<uint16_t>();
  if (a.mask != nullptr && s.group >= min_group) {
    switch (a.mask_dtype) {
      case SPECKV_BF16:
        return bf ? launch_sm100<__nv_bfloat16, 2, __nv_bfloat16>(mk, mv, s, stream)
                  : launch_sm100<__half, 2, __nv_bfloat16>(mk, mv, s, stream);
      case SPECKV_F16:
        return bf ? launch_sm100<__nv_bfloat16, 2, __half>(mk, mv, s, stream)
                  : launch_sm100<__half, 2, __half>(mk, mv, s, stream);
      default:
        return bf ? launch_sm100<__nv_bfloat16, 2, float>(mk, mv, s, stream)
                  : launch_sm100<__half, 2, float>(mk, mv, s, stream);
    }
  }
  switch (a.mask == nullptr ? SPECKV_F32 : a.mask_dtype) {
    case SPECKV_BF16:
      return bf ? launch_sm100<__nv_bfloat16, 1, __nv_bfloat16>(mk, mv, s, stream)
                : launch_sm100<__half, 1, __nv_bfloat16>(mk, mv, s, stream);
    case SPECKV_F16:
      return bf ? launch_sm100<__nv_bfloat16, 1, __half>(mk, mv, s, stream)
                : launch_sm100<__half, 1, __half>(mk, mv, s, stream);
    default:
      return bf ? launch_sm100<__nv_bfloat16, 1, float>(mk, mv, s, stream)
                : launch_sm100<__half, 1, float>(mk, mv, s, stream);
  }
}

}  // namespace speckv
