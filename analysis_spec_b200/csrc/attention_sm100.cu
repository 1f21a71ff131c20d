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
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t S_COL0 = 0, O_COL = 256;
constexpr unsigned long long kWaitNs = 2000000000ull;

// barrier slots (8 bytes each) after BAR_OFF
enum { B_KV_FULL = 0, B_KV_EMPTY = 2, B_S_FULL = 4, B_S_FREE = 6, B_P_FULL = 8, B_O_DONE = 9, B_Q_READY = 10,
       B_DRAIN = 11, B_ABORT = 12, TMEM_SLOT = 13 };

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
  unsigned long long* err;
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
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kWaitNs) {
        *abort_flag = 1;
        record_error(err, SPECKV_DERR_TIMEOUT, where);
        return false;
      }
    }
  }
}

// Time-bounded wait that ignores the abort flag: used to let in-flight asynchronous
// work finish before the CTA releases shared memory / TMEM.
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

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
// MODE 0: visibility bits; MODE 1: dense additive mask of type MT.
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
      // After an abort, copies still in flight must land before shared memory is released.
      if (*abort_flag) {
        for (int it = issued - 2 < 0 ? 0 : issued - 2; it < issued; ++it) drain_wait(bar(B_KV_FULL + (it & 1)), (it >> 1) & 1);
      }
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
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
        *reinterpret_cast<uint4*>(smem + Q_OFF + sw_chunk(t, c)) = v;
      }
      fence_proxy_async();
      mbar_arrive(bar(B_Q_READY));
    }
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

// 4-D map over a (batch, heads, len, 128) strided view: dims (d, len, heads, batch).
bool make_kv_map(CUtensorMap* map, const void* base, const long long* st, long long batch, long long heads,
                 long long len, int dtype) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)len, (cuuint64_t)heads, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)st[2] * 2, (cuuint64_t)st[1] * 2, (cuuint64_t)st[0] * 2};
  const cuuint32_t box[4] = {64, BN, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult res = fn(map, dtype == SPECKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS;
}

template <typename T, int MODE, typename MT>
int launch_sm100(const CUtensorMap& mk, const CUtensorMap& mv, const Sm100Args& s, cudaStream_t stream) {
  auto kern = attn_sm100_kernel<T, MODE, MT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
  const long long grid = (long long)s.batch * s.kv_heads * s.mtiles;
  kern<<<(unsigned)grid, kThreads, SMEM_BYTES, stream>>>(mk, mv, s);
  return check_launch("speckv_tree_attention(sm100)");
}

}  // namespace

bool sm100_supported(const AttnArgs& a) {
  if (a.dim != HD || (a.dtype != SPECKV_BF16 && a.dtype != SPECKV_F16)) return false;
  const long long* strides[3] = {a.qs, a.ks, a.vs};
  for (const long long* st : strides)
    for (int i = 0; i < 3; ++i)
      if ((st[i] * 2) % 16 != 0) return false;
  if (((uintptr_t)a.q | (uintptr_t)a.k | (uintptr_t)a.v | (uintptr_t)a.out) % 16 != 0) return false;
  if (a.batch > (1 << 20) || a.kv_len > (1 << 30)) return false;
  return true;
}

int attention_sm100(const AttnArgs& a, cudaStream_t stream) {
  const uint32_t* bits = a.bits;
  CUtensorMap mk, mv;
  if (!make_kv_map(&mk, a.k, a.ks, a.batch, a.kv_heads, a.kv_len, a.dtype) ||
      !make_kv_map(&mv, a.v, a.vs, a.batch, a.kv_heads, a.kv_len, a.dtype))
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
  s.err = err;
  const bool bf = a.dtype == SPECKV_BF16;
  if (bits != nullptr) {
    return bf ? launch_sm100<__nv_bfloat16, 0, float>(mk, mv, s, stream)
              : launch_sm100<__half, 0, float>(mk, mv, s, stream);
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
