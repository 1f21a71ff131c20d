// Tree-verify GQA attention, CUDA-core path for shapes the tensor-core kernel
// does not take (head dims other than 128, fp32 operands, tiny problems).
// Reads K/V once per query head straight from the strided cache views (no
// repeat_kv copy), applies the additive mask and an online softmax in fp32.
//
// Semantics: softmax(q k^T * scale + mask) v per (sequence, query head), with
// query head h reading KV head h / (q_heads / kv_heads), as transformers'
// sdpa_attention_forward (integrations/sdpa_attention.py:40-104) computes it.
#include "common.cuh"
#include "attention.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace speckv {
namespace {

constexpr int kRowsPerCta = 16;
constexpr int kCols = 32;
constexpr int kAttnThreads = 128;

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

template <typename T, typename M>
__global__ void __launch_bounds__(kAttnThreads) attn_generic_kernel(AttnArgs a) {
  extern __shared__ float sm[];
  const int D = (int)a.dim;
  float* Kt = sm;                        // [kCols][D + 1]
  float* Vt = Kt + kCols * (D + 1);      // [kCols][D]
  float* Qs = Vt + kCols * D;            // [kRowsPerCta][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long b = blockIdx.z, hq = blockIdx.y;
  const long long hk = hq / (a.q_heads / a.kv_heads);
  const long long r0 = (long long)blockIdx.x * kRowsPerCta;
  const T* q = static_cast<const T*>(a.q) + b * a.qs[0] + hq * a.qs[1];
  const T* k = static_cast<const T*>(a.k) + b * a.ks[0] + hk * a.ks[1];
  const T* v = static_cast<const T*>(a.v) + b * a.vs[0] + hk * a.vs[1];
  const M* mask = static_cast<const M*>(a.mask);
  for (int i = threadIdx.x; i < kRowsPerCta * D; i += kAttnThreads) {
    const long long r = r0 + i / D;
    Qs[i] = r < a.rows ? to_f<T>(q[r * a.qs[2] + i % D]) : 0.f;
  }
  constexpr int kMaxD = 8;  // D <= 256
  float o[4][kMaxD];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxD; ++j) o[i][j] = 0.f;
  }
  for (long long c0 = 0; c0 < a.kv_len; c0 += kCols) {
    __syncthreads();
    for (int i = threadIdx.x; i < kCols * D; i += kAttnThreads) {
      const int c = i / D, d = i % D;
      const long long col = c0 + c;
      Kt[c * (D + 1) + d] = col < a.kv_len ? to_f<T>(k[col * a.ks[2] + d]) : 0.f;
      Vt[c * D + d] = col < a.kv_len ? to_f<T>(v[col * a.vs[2] + d]) : 0.f;
    }
    __syncthreads();
    const long long col = c0 + lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rl = warp * 4 + i;
      const long long r = r0 + rl;
      if (r >= a.rows) continue;  // warp-uniform
      float s = -INFINITY;
      if (col < a.kv_len) {
        float acc = 0.f;
        const float* qr = Qs + rl * D;
        const float* kr = Kt + lane * (D + 1);
        for (int d = 0; d < D; ++d) acc = fmaf(qr[d], kr[d], acc);
        s = acc * a.scale;
        if (a.bits != nullptr) {
          const uint32_t w = a.bits[(b * a.rows + r) * a.row_words + (col >> 5)];
          if (!((w >> (col & 31)) & 1u)) s = -INFINITY;
        } else if (mask != nullptr) {
          s += to_f<M>(mask[(b * a.rows + r) * a.kv_len + col]);
        }
      }
      float tmax = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mnew = fmaxf(m[i], tmax);
      const float base = mnew == -INFINITY ? 0.f : mnew;  // rows with nothing visible yet stay at 0
      const float p = col < a.kv_len ? expf(s - base) : 0.f;
      const float corr = expf(m[i] - base);
      float psum = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l[i] = l[i] * corr + psum;
      m[i] = mnew;
#pragma unroll
      for (int j = 0; j < kMaxD; ++j) o[i][j] *= corr;
      for (int c = 0; c < kCols; ++c) {
        const float pc = __shfl_sync(0xffffffffu, p, c);
#pragma unroll
        for (int j = 0; j < kMaxD; ++j) {
          const int d = lane + 32 * j;
          if (d < D) o[i][j] = fmaf(pc, Vt[c * D + d], o[i][j]);
        }
      }
    }
  }
  T* out = static_cast<T*>(a.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long r = r0 + warp * 4 + i;
    if (r >= a.rows) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    T* orow = out + ((b * a.rows + r) * a.q_heads + hq) * a.dim;
#pragma unroll
    for (int j = 0; j < kMaxD; ++j) {
      const int d = lane + 32 * j;
      if (d < D) orow[d] = from_f<T>(o[i][j] * inv);
    }
  }
}

template <typename T>
int launch_typed(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = (size_t)(kCols * (a.dim + 1) + kCols * a.dim + kRowsPerCta * a.dim) * sizeof(float);
  dim3 grid((unsigned)((a.rows + kRowsPerCta - 1) / kRowsPerCta), (unsigned)a.q_heads, (unsigned)a.batch);
  switch (a.mask == nullptr ? -1 : a.mask_dtype) {
    case SPECKV_F32:
      cudaFuncSetAttribute(attn_generic_kernel<T, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attn_generic_kernel<T, float><<<grid, kAttnThreads, smem, s>>>(a);
      break;
    case SPECKV_F16:
      cudaFuncSetAttribute(attn_generic_kernel<T, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attn_generic_kernel<T, __half><<<grid, kAttnThreads, smem, s>>>(a);
      break;
    default:  // bf16 mask, or no mask (pointer is null and never read)
      cudaFuncSetAttribute(attn_generic_kernel<T, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attn_generic_kernel<T, __nv_bfloat16><<<grid, kAttnThreads, smem, s>>>(a);
      break;
  }
  return check_launch("speckv_tree_attention(generic)");
}

}  // namespace

int attention_generic(const AttnArgs& a, cudaStream_t s) {
  if (a.dim > 256) return fail(SPECKV_ENOSUPPORT, "speckv_tree_attention: head dim %lld above 256", a.dim);
  if (a.batch > 65535 || a.q_heads > 65535) return fail(SPECKV_ENOSUPPORT, "speckv_tree_attention: grid too large");
  switch (a.dtype) {
    case SPECKV_F32: return launch_typed<float>(a, s);
    case SPECKV_BF16: return launch_typed<__nv_bfloat16>(a, s);
    case SPECKV_F16: return launch_typed<__half>(a, s);
  }
  return fail(SPECKV_EINVAL, "speckv_tree_attention: unsupported dtype %d", a.dtype);
}

}  // namespace speckv
