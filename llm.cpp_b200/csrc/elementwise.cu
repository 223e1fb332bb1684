// HBM-bound kernels around the GEMMs and attention: LayerNorm fwd/bwd, GELU,
// residual, encoder (embedding gather / scatter), fused softmax + cross-
// entropy, AdamW, dtype casts.
//
// All kernels move 16-byte vectors with coalesced warp access and reduce
// with warp shuffles; cross-CTA reductions (LayerNorm dgamma/dbeta, loss
// mean) go through caller-provided scratch in a fixed order, so results are
// bitwise reproducible run to run.
//
// Reference kernels replaced: LayerNormForwardKernel / GammaAndBetaDerivate-
// Kernel / ComputeDerivateInputsKernel (gpt2/cuda/layernorm.cu:11-255),
// Gelu{Forward,Backward}Kernel (gelu.cu:13-48), Residual kernels
// (residual.cu:10-27), SoftmaxForwardKernel + CrossEntropy kernels
// (softmax.cu:13-91, cross_entropy.cu:7-32), Encoder kernels (encoder.cu:9-25),
// AdamWKernel (adamw.cu:8-33).
#include <algorithm>
#include <cmath>
#include <type_traits>

#include "ptx.cuh"
#include "runtime.h"

namespace llmk {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// 4 consecutive elements <-> float4
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
  float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__half* p, float4 v) {
  uint2 u;
  u.x = pack_f16x2(v.x, v.y);
  u.y = pack_f16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------ LayerNorm
// One warp per row; two-pass mean / variance as the reference CPU path
// (gpt2/layernorm.cpp:16-23). kV > 0: C == 128 * kV and the row stays in
// registers between the passes (one global read); kV == 0: any C % 4 == 0,
// the row is re-read from L1 for each pass.
template <typename OutT, int kV>
__global__ void __launch_bounds__(256) layernorm_fwd_kernel(OutT* __restrict__ out, float* __restrict__ mean,
                                                            float* __restrict__ rstd, const float* __restrict__ inp,
                                                            const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, int N, int C) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const float* x = inp + static_cast<long long>(row) * C;
  OutT* y = out + static_cast<long long>(row) * C;
  float m, r;
  if constexpr (kV > 0) {
    float4 v[kV];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      v[k] = ld4(x + lane * 4 + k * 128);
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    m = warp_sum(s) / C;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      float a = v[k].x - m, b = v[k].y - m, d = v[k].z - m, e = v[k].w - m;
      q += (a * a + b * b) + (d * d + e * e);
    }
    r = rsqrtf(warp_sum(q) / C + 1e-5f);
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const int c = lane * 4 + k * 128;
      float4 g = ld4(gamma + c), b = ld4(beta + c);
      st4(y + c, make_float4((v[k].x - m) * r * g.x + b.x, (v[k].y - m) * r * g.y + b.y,
                             (v[k].z - m) * r * g.z + b.z, (v[k].w - m) * r * g.w + b.w));
    }
  } else {
    float s = 0.f;
    for (int c = lane * 4; c < C; c += 128) {
      float4 v = ld4(x + c);
      s += (v.x + v.y) + (v.z + v.w);
    }
    m = warp_sum(s) / C;
    float q = 0.f;
    for (int c = lane * 4; c < C; c += 128) {
      float4 v = ld4(x + c);
      float a = v.x - m, b = v.y - m, d = v.z - m, e = v.w - m;
      q += (a * a + b * b) + (d * d + e * e);
    }
    r = rsqrtf(warp_sum(q) / C + 1e-5f);
    for (int c = lane * 4; c < C; c += 128) {
      float4 v = ld4(x + c), g = ld4(gamma + c), b = ld4(beta + c);
      st4(y + c, make_float4((v.x - m) * r * g.x + b.x, (v.y - m) * r * g.y + b.y, (v.z - m) * r * g.z + b.z,
                             (v.w - m) * r * g.w + b.w));
    }
  }
  if (lane == 0) {
    if (mean) mean[row] = m;
    if (rstd) rstd[row] = r;
  }
}

// dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat)) (gpt2/layernorm.cpp:60-69);
// dinp (+)= dx; optional bf16 copy of the new dinp. Each warp accumulates, for
// the rows it handles, dgamma (dy*xhat), dbeta (dy) and the column sums of the
// final dinp into its own smem slice [3][C]; the block then reduces the
// slices in warp order into partial[block][3][C]. kV as in the forward.
// Wide rows (kV >= 8, C >= 1024) hold 3 x kV float4 per lane and 96 KB+ of
// warp slices per block, so only one block fits an SM anyway: they get the
// whole register file instead of spilling under a two-blocks-per-SM bound.
template <typename DoutT, int kV>
__global__ void __launch_bounds__(256, (kV >= 8 ? 1 : 2)) layernorm_bwd_kernel(float* __restrict__ dinp, __nv_bfloat16* __restrict__ dinp_bf16,
                                                            float* __restrict__ partial, const DoutT* __restrict__ dout,
                                                            const float* __restrict__ inp,
                                                            const float* __restrict__ gamma,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ rstd, int N, int C,
                                                            int rows_per_block, int accumulate) {
  extern __shared__ float sm[];  // [warps][3][C]
  const int warps = blockDim.x / 32;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* dg = sm + static_cast<size_t>(w) * 3 * C;
  float* db = dg + C;
  float* ds = db + C;
  for (int c = lane; c < 3 * C; c += 32) dg[c] = 0.f;
  __syncwarp();
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(N, r0 + rows_per_block);
  for (int row = r0 + w; row < r1; row += warps) {
    const DoutT* dy = dout + static_cast<long long>(row) * C;
    const float* x = inp + static_cast<long long>(row) * C;
    float* dx = dinp + static_cast<long long>(row) * C;
    const float m = mean[row], r = rstd[row];
    float s1 = 0.f, s2 = 0.f;
    if constexpr (kV > 0) {
      float4 d[kV], xh[kV], old[kV];
      // every global read of the row issued together: one memory latency per row
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const int c = lane * 4 + k * 128;
        d[k] = ld4(dy + c);
        xh[k] = ld4(x + c);
        if (accumulate) old[k] = ld4(dx + c);
      }
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const int c = lane * 4 + k * 128;
        const float4 v = xh[k], g = ld4(gamma + c);
        xh[k] = make_float4((v.x - m) * r, (v.y - m) * r, (v.z - m) * r, (v.w - m) * r);
        float4 gd = make_float4(g.x * d[k].x, g.y * d[k].y, g.z * d[k].z, g.w * d[k].w);
        s1 += (gd.x + gd.y) + (gd.z + gd.w);
        s2 += (gd.x * xh[k].x + gd.y * xh[k].y) + (gd.z * xh[k].z + gd.w * xh[k].w);
      }
      s1 = warp_sum(s1) / C;
      s2 = warp_sum(s2) / C;
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const int c = lane * 4 + k * 128;
        float4 g = ld4(gamma + c);
        float4 o;
        o.x = r * ((g.x * d[k].x - xh[k].x * s2) - s1);
        o.y = r * ((g.y * d[k].y - xh[k].y * s2) - s1);
        o.z = r * ((g.z * d[k].z - xh[k].z * s2) - s1);
        o.w = r * ((g.w * d[k].w - xh[k].w * s2) - s1);
        if (accumulate) {
          o.x += old[k].x; o.y += old[k].y; o.z += old[k].z; o.w += old[k].w;
        }
        st4(dx + c, o);
        if (dinp_bf16) st4(dinp_bf16 + static_cast<long long>(row) * C + c, o);
        float4 a = ld4(dg + c), b = ld4(db + c), e = ld4(ds + c);
        st4(dg + c, make_float4(a.x + d[k].x * xh[k].x, a.y + d[k].y * xh[k].y, a.z + d[k].z * xh[k].z,
                                a.w + d[k].w * xh[k].w));
        st4(db + c, make_float4(b.x + d[k].x, b.y + d[k].y, b.z + d[k].z, b.w + d[k].w));
        st4(ds + c, make_float4(e.x + o.x, e.y + o.y, e.z + o.z, e.w + o.w));
      }
    } else {
      for (int c = lane * 4; c < C; c += 128) {
        float4 d = ld4(dy + c), v = ld4(x + c), g = ld4(gamma + c);
        float4 xh = make_float4((v.x - m) * r, (v.y - m) * r, (v.z - m) * r, (v.w - m) * r);
        float4 gd = make_float4(g.x * d.x, g.y * d.y, g.z * d.z, g.w * d.w);
        s1 += (gd.x + gd.y) + (gd.z + gd.w);
        s2 += (gd.x * xh.x + gd.y * xh.y) + (gd.z * xh.z + gd.w * xh.w);
        float4 a = ld4(dg + c), b = ld4(db + c);
        st4(dg + c, make_float4(a.x + d.x * xh.x, a.y + d.y * xh.y, a.z + d.z * xh.z, a.w + d.w * xh.w));
        st4(db + c, make_float4(b.x + d.x, b.y + d.y, b.z + d.z, b.w + d.w));
      }
      s1 = warp_sum(s1) / C;
      s2 = warp_sum(s2) / C;
      for (int c = lane * 4; c < C; c += 128) {
        float4 d = ld4(dy + c), v = ld4(x + c), g = ld4(gamma + c);
        float4 o;
        o.x = r * ((g.x * d.x - (v.x - m) * r * s2) - s1);
        o.y = r * ((g.y * d.y - (v.y - m) * r * s2) - s1);
        o.z = r * ((g.z * d.z - (v.z - m) * r * s2) - s1);
        o.w = r * ((g.w * d.w - (v.w - m) * r * s2) - s1);
        if (accumulate) {
          float4 p = ld4(dx + c);
          o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
        }
        st4(dx + c, o);
        if (dinp_bf16) st4(dinp_bf16 + static_cast<long long>(row) * C + c, o);
        float4 e = ld4(ds + c);
        st4(ds + c, make_float4(e.x + o.x, e.y + o.y, e.z + o.z, e.w + o.w));
      }
    }
  }
  __syncthreads();
  float* out = partial + static_cast<size_t>(blockIdx.x) * 3 * C;
  for (int c = threadIdx.x; c < 3 * C; c += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < warps; ++k) s += sm[static_cast<size_t>(k) * 3 * C + c];
    out[c] = s;
  }
}

// dst[c] (+)= sum over blocks of partial[b][c] for the 3C columns
// (dgamma | dbeta | dinp column sums), in block order: 32 columns x 8 block
// lanes per CTA, lanes combined in a fixed order.
__global__ void layernorm_bwd_reduce(float* __restrict__ dgamma, float* __restrict__ dbeta, float* __restrict__ dsum,
                                     const float* __restrict__ partial, int blocks, int C, int accumulate) {
  __shared__ float red[8][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < 3 * C)
    for (int b = threadIdx.y; b < blocks; b += 8) s += partial[static_cast<size_t>(b) * 3 * C + c];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || c >= 3 * C) return;
  float t = 0.f;
#pragma unroll
  for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
  if (c < C) {
    dgamma[c] = accumulate ? dgamma[c] + t : t;
  } else if (c < 2 * C) {
    dbeta[c - C] = accumulate ? dbeta[c - C] + t : t;
  } else if (dsum) {
    dsum[c - 2 * C] = t;
  }
}

// ------------------------------------------------------------ GELU / residual
template <typename T>
__global__ void gelu_fwd_kernel(T* __restrict__ out, const T* __restrict__ inp, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 v = ld4(inp + 4 * i);
    st4(out + 4 * i, make_float4(gelu_tanh(v.x), gelu_tanh(v.y), gelu_tanh(v.z), gelu_tanh(v.w)));
  }
}
template <typename T>
__global__ void gelu_bwd_kernel(T* __restrict__ dinp, const T* __restrict__ dout, const T* __restrict__ inp,
                                long long n4, int accumulate) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 x = ld4(inp + 4 * i), d = ld4(dout + 4 * i);
    float4 o = make_float4(d.x * gelu_tanh_grad(x.x), d.y * gelu_tanh_grad(x.y), d.z * gelu_tanh_grad(x.z),
                           d.w * gelu_tanh_grad(x.w));
    if (accumulate) {
      float4 p = ld4(dinp + 4 * i);
      o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
    }
    st4(dinp + 4 * i, o);
  }
}
template <typename T>
__global__ void add_kernel(T* __restrict__ out, const T* __restrict__ a, const T* __restrict__ b, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 x = ld4(a + 4 * i), y = ld4(b + 4 * i);
    st4(out + 4 * i, make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w));
  }
}
// residual backward: da (+)= dy; db (+)= dy (gpt2/cuda/residual.cu:17-27 accumulates)
template <typename T>
__global__ void residual_bwd_kernel(T* __restrict__ da, T* __restrict__ db, const T* __restrict__ dy, long long n4,
                                    int accumulate) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 d = ld4(dy + 4 * i);
    float4 a = d, b = d;
    if (accumulate) {
      float4 p = ld4(da + 4 * i), q = ld4(db + 4 * i);
      a = make_float4(p.x + d.x, p.y + d.y, p.z + d.z, p.w + d.w);
      b = make_float4(q.x + d.x, q.y + d.y, q.z + d.z, q.w + d.w);
    }
    st4(da + 4 * i, a);
    st4(db + 4 * i, b);
  }
}
template <typename Tin, typename Tout>
__global__ void cast_kernel(Tout* __restrict__ out, const Tin* __restrict__ in, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    st4(out + 4 * i, ld4(in + 4 * i));
}

// ------------------------------------------------------------ encoder
// out[b,t,:] = wte[tok[b,t],:] + wpe[t,:] (gpt2/encoder.cpp:5-20)
__global__ void encoder_fwd_kernel(float* __restrict__ out, const int* __restrict__ tokens,
                                   const float* __restrict__ wte, const float* __restrict__ wpe, int BT, int T, int C) {
  const int c4 = C / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < static_cast<long long>(BT) * c4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int bt = static_cast<int>(i / c4), c = static_cast<int>(i - static_cast<long long>(bt) * c4) * 4;
    const int t = bt % T;
    float4 e = ld4(wte + static_cast<long long>(tokens[bt]) * C + c), p = ld4(wpe + static_cast<long long>(t) * C + c);
    st4(out + static_cast<long long>(bt) * C + c, make_float4(e.x + p.x, e.y + p.y, e.z + p.z, e.w + p.w));
  }
}
// dwpe[t,:] += sum_b dout[b,t,:] in batch order (deterministic).
__global__ void encoder_bwd_wpe_kernel(float* __restrict__ dwpe, const float* __restrict__ dout, int B, int T, int C) {
  // four columns a thread, four batch rows' loads in flight; the sum still
  // runs over b in order
  const long long n = static_cast<long long>(T) * C, n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float* p = dout + 4 * i;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    int b = 0;
    for (; b + 4 <= B; b += 4) {
      float4 d[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) d[k] = ld4(p + static_cast<long long>(b + k) * n);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s.x += d[k].x; s.y += d[k].y; s.z += d[k].z; s.w += d[k].w;
      }
    }
    for (; b < B; ++b) {
      const float4 d = ld4(p + static_cast<long long>(b) * n);
      s.x += d.x; s.y += d.y; s.z += d.z; s.w += d.w;
    }
    const float4 o = ld4(dwpe + 4 * i);
    st4(dwpe + 4 * i, make_float4(o.x + s.x, o.y + s.y, o.z + s.z, o.w + s.w));
  }
}
// dwte[tok,:] += dout[b,t,:]: positions sharing a token are summed in
// position order by one thread per (first position of that token, column)
// using the per-position "next with same token" links built on the host side
// of the call (see encoder_backward); positions that are not the first of
// their token do nothing.
__global__ void encoder_bwd_wte_kernel(float* __restrict__ dwte, const float* __restrict__ dout,
                                       const int* __restrict__ tokens, const int* __restrict__ first_of,
                                       const int* __restrict__ next_same, int BT, int C) {
  const int c4 = C / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < static_cast<long long>(BT) * c4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int bt = static_cast<int>(i / c4), c = static_cast<int>(i - static_cast<long long>(bt) * c4) * 4;
    if (!first_of[bt]) continue;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = bt; p >= 0; p = next_same[p]) {
      float4 d = ld4(dout + static_cast<long long>(p) * C + c);
      s.x += d.x; s.y += d.y; s.z += d.z; s.w += d.w;
    }
    float* dst = dwte + static_cast<long long>(tokens[bt]) * C + c;
    float4 o = ld4(dst);
    st4(dst, make_float4(o.x + s.x, o.y + s.y, o.z + s.z, o.w + s.w));
  }
}
// Sorts the keys (token << 15 | position) of BT <= 32768 positions with a
// bitonic network in one CTA's shared memory (n = next power of two >= BT,
// padded with 0xFFFFFFFF). Equal tokens end up adjacent, positions ascending.
constexpr int kSortMaxBT = 32768;
__global__ void __launch_bounds__(1024) encoder_sort_kernel(unsigned int* __restrict__ sorted,
                                                            const int* __restrict__ tokens, int BT, int n) {
  extern __shared__ unsigned int key[];
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    key[i] = i < BT ? (static_cast<unsigned int>(tokens[i]) << 15) | static_cast<unsigned int>(i) : 0xFFFFFFFFu;
  __syncthreads();
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned int a = key[i], b = key[ixj];
          const bool ascending = (i & k) == 0;
          if ((a > b) == ascending) {
            key[i] = b;
            key[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < BT; i += blockDim.x) sorted[i] = key[i];
}
// The same network for n = kPer * 1024 keys, with the stages whose partner
// distance j is below kPer run in registers on each thread's kPer
// consecutive keys (one shared-memory round trip and one barrier per merge
// size instead of one per stage). Shared memory holds one pad word per 32
// keys, so the threads' strided register loads and the passes' consecutive
// accesses both avoid bank conflicts.
__device__ __forceinline__ int sort_pad(int i) { return i + (i >> 5); }

template <int kPer>
__global__ void __launch_bounds__(1024) encoder_sort_reg_kernel(unsigned int* __restrict__ sorted,
                                                                const int* __restrict__ tokens, int BT) {
  constexpr int n = kPer * 1024;
  extern __shared__ unsigned int key[];  // n + n / 32 words
  for (int i = threadIdx.x; i < n; i += 1024)
    key[sort_pad(i)] = i < BT ? (static_cast<unsigned int>(tokens[i]) << 15) | static_cast<unsigned int>(i) : 0xFFFFFFFFu;
  __syncthreads();
  const int base = threadIdx.x * kPer;
  unsigned int r[kPer];
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j >= kPer; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += 1024) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned int a = key[sort_pad(i)], b = key[sort_pad(ixj)];
          const bool ascending = (i & k) == 0;
          if ((a > b) == ascending) {
            key[sort_pad(i)] = b;
            key[sort_pad(ixj)] = a;
          }
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int e = 0; e < kPer; ++e) r[e] = key[sort_pad(base + e)];
#pragma unroll
    for (int j = kPer / 2; j > 0; j >>= 1) {
      if (j < k) {
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          if ((e & j) == 0) {
            const int f = e | j;
            const bool ascending = ((base + e) & k) == 0;
            const unsigned int a = r[e], b = r[f];
            if ((a > b) == ascending) {
              r[e] = b;
              r[f] = a;
            }
          }
        }
      }
    }
#pragma unroll
    for (int e = 0; e < kPer; ++e) key[sort_pad(base + e)] = r[e];
    __syncthreads();
  }
  for (int i = threadIdx.x; i < BT; i += 1024) sorted[i] = key[sort_pad(i)];
}

// The same sorted keys for BT <= 16384 and tokens below 2^16, by a stable
// LSD radix sort on the token in one CTA: two passes of one 8-bit digit. A
// pass counts each warp's digits (warp w owns 512-or-fewer consecutive keys),
// scans the counts in (digit, warp) order into every warp's first slot per
// digit, and lets each warp scatter its keys in order, 32 a round, ranking
// equal digits inside a round by lane (match.any). Equal tokens therefore keep
// their position order, and since the keys are distinct the result is the
// bitonic network's array, in a few microseconds instead of ~100.
constexpr int kRadixMaxBT = 16384;
// digit counters [256 digits][32 warps] with a row stride of 33 words, so the
// 32 lanes of a warp (one warp column, different digits) hit different banks
constexpr int kRadixRow = 33;
constexpr size_t kRadixSmem = (2 * kRadixMaxBT + 256 * kRadixRow + 32) * sizeof(unsigned int);
__global__ void __launch_bounds__(1024) encoder_radix_kernel(unsigned int* __restrict__ sorted,
                                                             const int* __restrict__ tokens, int BT) {
  extern __shared__ unsigned int rsm[];
  unsigned int* src = rsm;                     // keys, kRadixMaxBT
  unsigned int* dst = rsm + kRadixMaxBT;       // keys, kRadixMaxBT
  unsigned int* cnt = rsm + 2 * kRadixMaxBT;   // [256 digits][32 warps] (row stride 33), then 32 warp totals
  unsigned int* wsum = cnt + 256 * kRadixRow;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned int lt = (1u << lane) - 1u;
  for (int i = tid; i < BT; i += 1024) src[i] = (static_cast<unsigned int>(tokens[i]) << 15) | static_cast<unsigned int>(i);
  const int per = (BT + 31) / 32;
  const int w0 = min(BT, warp * per), w1 = min(BT, w0 + per);
  for (int pass = 0; pass < 2; ++pass) {
    const int shift = 15 + 8 * pass;
    for (int i = tid; i < 256 * kRadixRow; i += 1024) cnt[i] = 0;
    __syncthreads();
    for (int i = w0 + lane; i < w1; i += 32) atomicAdd(&cnt[((src[i] >> shift) & 255u) * kRadixRow + warp], 1u);
    __syncthreads();
    // exclusive scan of the 8192 counts: 8 consecutive per thread, then the
    // thread totals across the block
    // entry e = 8 tid + k is (digit e / 32, warp e % 32)
    const int crow = (tid >> 2) * kRadixRow + (tid & 3) * 8;
    unsigned int c8[8], run = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      c8[k] = run;
      run += cnt[crow + k];
    }
    unsigned int inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      unsigned int v = wsum[lane], vi = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, vi, o);
        if (lane >= o) vi += y;
      }
      wsum[lane] = vi - v;  // exclusive
    }
    __syncthreads();
    const unsigned int base = wsum[warp] + inc - run;
#pragma unroll
    for (int k = 0; k < 8; ++k) cnt[crow + k] = base + c8[k];
    __syncthreads();
    // stable scatter, 32 keys of this warp a round
    for (int b0 = w0; b0 < w1; b0 += 32) {
      const int i = b0 + lane;
      const bool valid = i < w1;
      const unsigned int key = valid ? src[i] : 0u;
      const unsigned int d = valid ? (key >> shift) & 255u : 256u + static_cast<unsigned int>(lane);
      const unsigned int peers = __match_any_sync(0xffffffffu, d);
      unsigned int slot = 0;
      if (valid) slot = cnt[d * kRadixRow + warp] + __popc(peers & lt);
      __syncwarp();
      if (valid) {
        dst[slot] = key;
        if ((peers >> lane) == 1u) cnt[d * kRadixRow + warp] = slot + 1;  // the group's last lane advances the slot
      }
      __syncwarp();
    }
    __syncthreads();
    unsigned int* t = src;
    src = dst;
    dst = t;
  }
  for (int i = tid; i < BT; i += 1024) sorted[i] = src[i];
}

// dwte[tok,:] += sum of dout rows of the positions holding tok, in position
// order: the first sorted key of each run of equal tokens sums its run.
// Runs longer than this many positions (frequent tokens) are summed by
// encoder_bwd_wte_long_kernel in 32 ordered segments instead of one thread's
// sequential loop.
constexpr int kLongRun = 64;

__global__ void encoder_bwd_wte_sorted_kernel(float* __restrict__ dwte, const float* __restrict__ dout,
                                              const unsigned int* __restrict__ sorted, int BT, int C,
                                              int* __restrict__ long_runs) {
  const int c4 = C / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < static_cast<long long>(BT) * c4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int idx = static_cast<int>(i / c4), c = static_cast<int>(i - static_cast<long long>(idx) * c4) * 4;
    const unsigned int tok = sorted[idx] >> 15;
    if (idx > 0 && (sorted[idx - 1] >> 15) == tok) continue;
    if (idx + kLongRun < BT && (sorted[idx + kLongRun] >> 15) == tok) {
      // a long run: listed once (by its first column group) for the segmented kernel
      if (c == 0) long_runs[1 + atomicAdd(long_runs, 1)] = idx;
      continue;
    }
    // the run's rows added in position order, their loads in flight together:
    // eight for the first block (most runs are short), 32 a block after that
    // (frequent tokens make runs of thousands)
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    bool more = true;
    int j = idx;
    auto block = [&](auto ku) {
      constexpr int kU = decltype(ku)::value;
      unsigned int key[kU];
      bool in[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        key[u] = j + u < BT ? sorted[j + u] : 0xFFFFFFFFu;
        in[u] = (key[u] >> 15) == tok;
      }
      float4 d[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        d[u] = in[u] ? ld4(dout + static_cast<long long>(key[u] & 0x7FFFu) * C + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (in[u]) {
          s.x += d[u].x; s.y += d[u].y; s.z += d[u].z; s.w += d[u].w;
        }
      more = in[kU - 1];
      j += kU;
    };
    block(std::integral_constant<int, 8>{});
    while (more) block(std::integral_constant<int, 32>{});
    float* dst = dwte + static_cast<long long>(tok) * C + c;
    float4 o = ld4(dst);
    st4(dst, make_float4(o.x + s.x, o.y + s.y, o.z + s.z, o.w + s.w));
  }
}

// dwte[tok,:] += the sum of one long run's dout rows (more than kLongRun
// positions): a block per 128-column chunk and run of the list (blocks
// stride over the runs); warp w sums the w-th of 32 equal contiguous segments
// of the run in position order, and warp 0 adds the 32 segment sums in
// segment order. Fixed segmentation and order:
// the result is the same on every run (not the strictly sequential sum a
// short run gets).
__global__ void __launch_bounds__(1024) encoder_bwd_wte_long_kernel(float* __restrict__ dwte,
                                                                    const float* __restrict__ dout,
                                                                    const unsigned int* __restrict__ sorted, int BT,
                                                                    int C, const int* __restrict__ long_runs) {
  __shared__ float4 part[32][32];
  __shared__ int run_end;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.y * 128 + lane * 4;
  const int nruns = long_runs[0];
  for (int r = blockIdx.x; r < nruns; r += gridDim.x) {
    const int rs = long_runs[1 + r];
    const unsigned int tok = sorted[rs] >> 15;
    if (threadIdx.x == 0) {
      // first index past the run: binary search over the sorted keys
      int lo = rs + 1, hi = BT;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((sorted[mid] >> 15) == tok) lo = mid + 1;
        else hi = mid;
      }
      run_end = lo;
    }
    __syncthreads();
    const int len = run_end - rs, seg = (len + 31) / 32;
    const int j0 = rs + min(len, warp * seg), j1 = rs + min(len, (warp + 1) * seg);
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < C) {
      int j = j0;
      for (; j + 8 <= j1; j += 8) {
        float4 d[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) d[u] = ld4(dout + static_cast<long long>(sorted[j + u] & 0x7FFFu) * C + c);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          s.x += d[u].x; s.y += d[u].y; s.z += d[u].z; s.w += d[u].w;
        }
      }
      for (; j < j1; ++j) {
        const float4 d = ld4(dout + static_cast<long long>(sorted[j] & 0x7FFFu) * C + c);
        s.x += d.x; s.y += d.y; s.z += d.z; s.w += d.w;
      }
    }
    part[warp][lane] = s;
    __syncthreads();
    if (warp == 0 && c < C) {
      float4 t = part[0][lane];
#pragma unroll 1
      for (int w = 1; w < 32; ++w) {
        const float4 p = part[w][lane];
        t.x += p.x; t.y += p.y; t.z += p.z; t.w += p.w;
      }
      float* dst = dwte + static_cast<long long>(tok) * C + c;
      const float4 o = ld4(dst);
      st4(dst, make_float4(o.x + t.x, o.y + t.y, o.z + t.z, o.w + t.w));
    }
    __syncthreads();  // part and run_end are rewritten for the next run
  }
}

// Builds first_of / next_same on the device: for each position, the next
// later position holding the same token (or -1), and whether no earlier
// position holds it. O(BT * window) scan per position, bounded by BT.
__global__ void encoder_links_kernel(int* __restrict__ first_of, int* __restrict__ next_same,
                                     const int* __restrict__ tokens, int BT) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= BT) return;
  const int tok = tokens[p];
  int nxt = -1;
  for (int q = p + 1; q < BT; ++q)
    if (tokens[q] == tok) { nxt = q; break; }
  int first = 1;
  for (int q = p - 1; q >= 0; --q)
    if (tokens[q] == tok) { first = 0; break; }
  next_same[p] = nxt;
  first_of[p] = first;
}

// ------------------------------------------------- softmax + cross-entropy
// One CTA per row of logits[BT, ld] (first V columns live): loss[row] =
// logsumexp - logit[target]; when dlogits != NULL, dlogits = (softmax -
// onehot) * dscale on columns < V and 0 on [V, ld) (the reference's
// CrossEntropySoftmaxBackward with scale 1/(B*T), gpt2/cuda/gpt2cuda.cu:398).
// dlogits may alias logits.
// kSoftmaxOnly: no targets or losses; `dlogits` receives softmax on the
// columns < V, and [V, ld) is left untouched (the reference's
// BatchSoftmaxForward, gpt2/cuda/softmax.cu:13-91, writes only the first V).
template <typename T, bool kSoftmaxOnly = false>
__global__ void __launch_bounds__(512) softmax_xent_kernel(float* __restrict__ losses, T* dlogits, const T* logits,
                                                           const int* __restrict__ targets, int V, int ld,
                                                           float dscale) {
  const long long row = blockIdx.x;
  const T* x = logits + row * ld;
  __shared__ float red[32];
  __shared__ float bcast[2];
  const int tid = threadIdx.x, nt = blockDim.x;
  const int v4 = V / 4;  // vectorised part; tail handled scalar
  // pass 1: online max / sum
  float m = -INFINITY, s = 0.f;
  for (int i = tid; i < v4; i += nt) {
    float4 v = ld4(x + 4 * i);
    float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    if (mx > m) {
      s *= __expf(m - mx);
      m = mx;
    }
    s += __expf(v.x - m) + __expf(v.y - m) + __expf(v.z - m) + __expf(v.w - m);
  }
  for (int i = 4 * v4 + tid; i < V; i += nt) {
    float v = to_f(x[i]);
    if (v > m) {
      s *= __expf(m - v);
      m = v;
    }
    s += __expf(v - m);
  }
  // block reduce (max, then rescaled sum)
  float bm = warp_max(m);
  if ((tid & 31) == 0) red[tid >> 5] = bm;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (nt >> 5) ? red[tid] : -INFINITY;
    v = warp_max(v);
    if (tid == 0) bcast[0] = v;
  }
  __syncthreads();
  const float M = bcast[0];
  float ss = (m == -INFINITY) ? 0.f : s * __expf(m - M);
  ss = warp_sum(ss);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (nt >> 5) ? red[tid] : 0.f;
    v = warp_sum(v);
    if (tid == 0) bcast[1] = v;
  }
  __syncthreads();
  const float S = bcast[1];
  const float inv = 1.0f / S;
  if constexpr (kSoftmaxOnly) {
    T* d = dlogits + row * ld;
    for (int i = tid; i < v4; i += nt) {
      float4 v = ld4(x + 4 * i);
      st4(d + 4 * i, make_float4(__expf(v.x - M) * inv, __expf(v.y - M) * inv, __expf(v.z - M) * inv,
                                 __expf(v.w - M) * inv));
    }
    for (int i = 4 * v4 + tid; i < V; i += nt) {
      const float g = __expf(to_f(x[i]) - M) * inv;
      if constexpr (sizeof(T) == 4) d[i] = g;
      else d[i] = __float2bfloat16(g);
    }
    return;
  }
  const int tgt = targets[row];
  const float lse = M + logf(S);
  if (tid == 0) losses[row] = lse - to_f(x[tgt]);
  if (dlogits == nullptr) return;
  T* d = dlogits + row * ld;
  for (int i = tid; i < v4; i += nt) {
    float4 v = ld4(x + 4 * i);
    float4 p = make_float4(__expf(v.x - M) * inv, __expf(v.y - M) * inv, __expf(v.z - M) * inv,
                           __expf(v.w - M) * inv);
    const int c = 4 * i;
    if (tgt >= c && tgt < c + 4) {
      if (tgt == c) p.x -= 1.f;
      else if (tgt == c + 1) p.y -= 1.f;
      else if (tgt == c + 2) p.z -= 1.f;
      else p.w -= 1.f;
    }
    st4(d + c, make_float4(p.x * dscale, p.y * dscale, p.z * dscale, p.w * dscale));
  }
  for (int i = 4 * v4 + tid; i < ld; i += nt) {
    float g = 0.f;
    if (i < V) g = (__expf(to_f(x[i]) - M) * inv - (i == tgt ? 1.f : 0.f)) * dscale;
    if constexpr (sizeof(T) == 4) d[i] = g;
    else d[i] = __float2bfloat16(g);
  }
}

// losses[row] (+)= -log(probs[row, targets[row]]) — the reference's
// CrossEntropyForward over probabilities (gpt2/cuda/cross_entropy.cu:24-29,
// which accumulates). A target outside [0, ld) gives NaN for that row.
template <typename T>
__global__ void xent_from_probs_kernel(float* __restrict__ losses, const T* __restrict__ probs,
                                       const int* __restrict__ targets, int rows, int ld, int accumulate) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int t = targets[r];
  const float l = (t >= 0 && t < ld) ? -logf(to_f(probs[static_cast<long long>(r) * ld + t])) : __int_as_float(0x7fc00000);
  losses[r] = accumulate ? losses[r] + l : l;
}

// dlogits[row, c] = (accumulate ? dlogits[row, c] : 0) + (probs[row, c] -
// [c == target]) * scale on the columns c < V; [V, ld) untouched.
template <typename T>
__global__ void xent_softmax_backward_kernel(T* __restrict__ dlogits, const T* __restrict__ probs,
                                             const int* __restrict__ targets, int V, int ld, float scale,
                                             int accumulate) {
  const long long row = blockIdx.y;
  const int t = targets[row];
  const T* p = probs + row * ld;
  T* d = dlogits + row * ld;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < V; c += gridDim.x * blockDim.x) {
    float g = (to_f(p[c]) - (c == t ? 1.f : 0.f)) * scale;
    if (accumulate) g += to_f(d[c]);
    if constexpr (sizeof(T) == 4) d[c] = g;
    else d[c] = __float2bfloat16(g);
  }
}

// mean of losses[n] (fixed-order tree in one CTA)
__global__ void mean_kernel(float* __restrict__ out, const float* __restrict__ x, int n) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) *out = v / n;
  }
}

// ------------------------------------------------------------ AdamW
// p -= lr * (mhat / (sqrt(vhat) + eps) + wd * p) (gpt2/cuda/adamw.cu:18-30);
// g is scaled by grad_scale on the fly (1/world for data-parallel averaging);
// p_bf16 (optional) receives the updated parameters rounded to bf16. The
// hyperparameters come as kernel arguments, or (hp_dev != nullptr) from
// device memory, so a captured CUDA graph replays with per-step values.
struct AdamHP {
  float lr, b1, b2, eps, wd, inv_c1, inv_c2, grad_scale;
};
__global__ void adamw_kernel(float* __restrict__ p, __nv_bfloat16* __restrict__ p_bf16, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, long long n4, AdamHP hp_arg,
                             const AdamHP* __restrict__ hp_dev) {
  const AdamHP hp = hp_dev ? *hp_dev : hp_arg;
  const float lr = hp.lr, b1 = hp.b1, b2 = hp.b2, eps = hp.eps, wd = hp.wd, inv_c1 = hp.inv_c1, inv_c2 = hp.inv_c2,
              grad_scale = hp.grad_scale;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 pp = ld4(p + 4 * i), gg = ld4(g + 4 * i), mm = ld4(m + 4 * i), vv = ld4(v + 4 * i);
    float pa[4] = {pp.x, pp.y, pp.z, pp.w}, ga[4] = {gg.x, gg.y, gg.z, gg.w}, ma[4] = {mm.x, mm.y, mm.z, mm.w},
          va[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = ga[k] * grad_scale;
      const float m_ = b1 * ma[k] + (1.f - b1) * gr;
      const float v_ = b2 * va[k] + (1.f - b2) * gr * gr;
      ma[k] = m_;
      va[k] = v_;
      pa[k] -= lr * ((m_ * inv_c1) / (sqrtf(v_ * inv_c2) + eps) + wd * pa[k]);
    }
    st4(p + 4 * i, make_float4(pa[0], pa[1], pa[2], pa[3]));
    st4(m + 4 * i, make_float4(ma[0], ma[1], ma[2], ma[3]));
    st4(v + 4 * i, make_float4(va[0], va[1], va[2], va[3]));
    if (p_bf16) st4(p_bf16 + 4 * i, make_float4(pa[0], pa[1], pa[2], pa[3]));
  }
}

int grid_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(b, num_sms() * 16LL)));
}

int ln_bwd_blocks(int N) { return std::max(1, std::min(2 * num_sms(), (N + 7) / 8)); }

}  // namespace
}  // namespace llmk

using namespace llmk;

static bool a16(const void* p) { return p == nullptr || aligned16(p); }

extern "C" {

}  // extern "C"

template <typename OutT>
static void ln_fwd_dispatch(OutT* out, float* mean, float* rstd, const float* inp, const float* gamma,
                            const float* beta, int N, int C, cudaStream_t s) {
  const int grid = (N + 7) / 8;
  switch (C % 128 ? 0 : C / 128) {
    case 4: layernorm_fwd_kernel<OutT, 4><<<grid, 256, 0, s>>>(out, mean, rstd, inp, gamma, beta, N, C); break;
    case 6: layernorm_fwd_kernel<OutT, 6><<<grid, 256, 0, s>>>(out, mean, rstd, inp, gamma, beta, N, C); break;
    case 8: layernorm_fwd_kernel<OutT, 8><<<grid, 256, 0, s>>>(out, mean, rstd, inp, gamma, beta, N, C); break;
    case 10: layernorm_fwd_kernel<OutT, 10><<<grid, 256, 0, s>>>(out, mean, rstd, inp, gamma, beta, N, C); break;
    case 12: layernorm_fwd_kernel<OutT, 12><<<grid, 256, 0, s>>>(out, mean, rstd, inp, gamma, beta, N, C); break;
    default: layernorm_fwd_kernel<OutT, 0><<<grid, 256, 0, s>>>(out, mean, rstd, inp, gamma, beta, N, C); break;
  }
}

extern "C" {

int llmk_layernorm_forward(void* out, llmk_dtype out_dtype, float* mean, float* rstd, const float* inp,
                           const float* gamma, const float* beta, int N, int C, void* stream) {
  if (!out || !inp || !gamma || !beta || N <= 0 || C <= 0) return fail(LLMK_ERR_INVALID_ARG, "layernorm_forward");
  if (C % 4 || !a16(out) || !a16(inp) || !a16(gamma) || !a16(beta))
    return fail(LLMK_ERR_UNSUPPORTED, "layernorm_forward: C % 4 == 0 and 16-byte alignment required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (out_dtype == LLMK_BF16)
    ln_fwd_dispatch(static_cast<__nv_bfloat16*>(out), mean, rstd, inp, gamma, beta, N, C, s);
  else
    ln_fwd_dispatch(static_cast<float*>(out), mean, rstd, inp, gamma, beta, N, C, s);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

size_t llmk_layernorm_backward_workspace(int N, int C) {
  if (N <= 0 || C <= 0) return 0;
  return static_cast<size_t>(ln_bwd_blocks(N)) * 3 * C * sizeof(float);
}

}  // extern "C"

template <typename DoutT, int kV>
static int ln_bwd_launch(int blocks, size_t smem, cudaStream_t s, float* dinp, __nv_bfloat16* dinp_bf16, float* part,
                         const DoutT* dout, const float* inp, const float* gamma, const float* mean, const float* rstd,
                         int N, int C, int rows_per_block, int acc_in) {
  auto k = layernorm_bwd_kernel<DoutT, kV>;
  LLMK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  k<<<blocks, 256, smem, s>>>(dinp, dinp_bf16, part, dout, inp, gamma, mean, rstd, N, C, rows_per_block, acc_in);
  return LLMK_OK;
}

template <typename DoutT>
static int ln_bwd_dispatch(int blocks, size_t smem, cudaStream_t s, float* dinp, __nv_bfloat16* dinp_bf16,
                           float* part, const DoutT* dout, const float* inp, const float* gamma, const float* mean,
                           const float* rstd, int N, int C, int rows_per_block, int acc_in) {
  switch (C % 128 ? 0 : C / 128) {
    case 4: return ln_bwd_launch<DoutT, 4>(blocks, smem, s, dinp, dinp_bf16, part, dout, inp, gamma, mean, rstd, N, C, rows_per_block, acc_in);
    case 6: return ln_bwd_launch<DoutT, 6>(blocks, smem, s, dinp, dinp_bf16, part, dout, inp, gamma, mean, rstd, N, C, rows_per_block, acc_in);
    case 8: return ln_bwd_launch<DoutT, 8>(blocks, smem, s, dinp, dinp_bf16, part, dout, inp, gamma, mean, rstd, N, C, rows_per_block, acc_in);
    case 10: return ln_bwd_launch<DoutT, 10>(blocks, smem, s, dinp, dinp_bf16, part, dout, inp, gamma, mean, rstd, N, C, rows_per_block, acc_in);
    default: return ln_bwd_launch<DoutT, 0>(blocks, smem, s, dinp, dinp_bf16, part, dout, inp, gamma, mean, rstd, N, C, rows_per_block, acc_in);
  }
}

extern "C" {

int llmk_layernorm_backward(float* dinp, void* dinp_bf16, float* dgamma, float* dbeta, float* dinp_colsum,
                            const void* dout, llmk_dtype dout_dtype, const float* inp, const float* gamma,
                            const float* mean, const float* rstd, int N, int C, int flags, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!dinp || !dgamma || !dbeta || !dout || !inp || !gamma || !mean || !rstd || N <= 0 || C <= 0)
    return fail(LLMK_ERR_INVALID_ARG, "layernorm_backward");
  if (C % 4 || !a16(dinp) || !a16(dinp_bf16) || !a16(dout) || !a16(inp) || !a16(gamma))
    return fail(LLMK_ERR_UNSUPPORTED, "layernorm_backward: C % 4 == 0 and 16-byte alignment required");
  const int blocks = ln_bwd_blocks(N);
  if (!workspace || workspace_bytes < static_cast<size_t>(blocks) * 3 * C * sizeof(float))
    return fail(LLMK_ERR_WORKSPACE, "layernorm_backward: workspace too small");
  const size_t smem = static_cast<size_t>(8) * 3 * C * sizeof(float);
  if (smem > 220 * 1024) return fail(LLMK_ERR_UNSUPPORTED, "layernorm_backward: C too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rows_per_block = (N + blocks - 1) / blocks;
  float* part = static_cast<float*>(workspace);
  const int acc_in = (flags & LLMK_ACCUM_DINP) ? 1 : 0;
  if (dout_dtype == LLMK_BF16)
    LLMK_TRY(ln_bwd_dispatch(blocks, smem, s, dinp, static_cast<__nv_bfloat16*>(dinp_bf16), part,
                             static_cast<const __nv_bfloat16*>(dout), inp, gamma, mean, rstd, N, C, rows_per_block,
                             acc_in));
  else
    LLMK_TRY(ln_bwd_dispatch(blocks, smem, s, dinp, static_cast<__nv_bfloat16*>(dinp_bf16), part,
                             static_cast<const float*>(dout), inp, gamma, mean, rstd, N, C, rows_per_block, acc_in));
  layernorm_bwd_reduce<<<(3 * C + 31) / 32, dim3(32, 8), 0, s>>>(dgamma, dbeta, dinp_colsum, part, blocks, C,
                                                                 (flags & LLMK_ACCUM_DPARAM) ? 1 : 0);
  count_launch(2);
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_gelu_forward(void* out, const void* inp, llmk_dtype dtype, long long n, void* stream) {
  if (!out || !inp || n < 0) return fail(LLMK_ERR_INVALID_ARG, "gelu_forward");
  if (n % 4 || !a16(out) || !a16(inp)) return fail(LLMK_ERR_UNSUPPORTED, "gelu_forward: n % 4, alignment");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LLMK_BF16)
    gelu_fwd_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(static_cast<__nv_bfloat16*>(out),
                                                         static_cast<const __nv_bfloat16*>(inp), n / 4);
  else
    gelu_fwd_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(static_cast<float*>(out), static_cast<const float*>(inp),
                                                         n / 4);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_gelu_backward(void* dinp, const void* dout, const void* inp, llmk_dtype dtype, long long n, int accumulate,
                       void* stream) {
  if (!dinp || !dout || !inp || n < 0) return fail(LLMK_ERR_INVALID_ARG, "gelu_backward");
  if (n % 4 || !a16(dinp) || !a16(dout) || !a16(inp)) return fail(LLMK_ERR_UNSUPPORTED, "gelu_backward: n % 4");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LLMK_BF16)
    gelu_bwd_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(
        static_cast<__nv_bfloat16*>(dinp), static_cast<const __nv_bfloat16*>(dout),
        static_cast<const __nv_bfloat16*>(inp), n / 4, accumulate);
  else
    gelu_bwd_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(static_cast<float*>(dinp), static_cast<const float*>(dout),
                                                         static_cast<const float*>(inp), n / 4, accumulate);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_residual_forward(void* out, const void* a, const void* b, llmk_dtype dtype, long long n, void* stream) {
  if (!out || !a || !b || n < 0) return fail(LLMK_ERR_INVALID_ARG, "residual_forward");
  if (n % 4 || !a16(out) || !a16(a) || !a16(b)) return fail(LLMK_ERR_UNSUPPORTED, "residual_forward: n % 4");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LLMK_BF16)
    add_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(static_cast<__nv_bfloat16*>(out),
                                                    static_cast<const __nv_bfloat16*>(a),
                                                    static_cast<const __nv_bfloat16*>(b), n / 4);
  else
    add_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(static_cast<float*>(out), static_cast<const float*>(a),
                                                    static_cast<const float*>(b), n / 4);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_residual_backward(void* da, void* db, const void* dy, llmk_dtype dtype, long long n, int accumulate,
                           void* stream) {
  if (!da || !db || !dy || n < 0) return fail(LLMK_ERR_INVALID_ARG, "residual_backward");
  if (n % 4 || !a16(da) || !a16(db) || !a16(dy)) return fail(LLMK_ERR_UNSUPPORTED, "residual_backward: n % 4");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LLMK_BF16)
    residual_bwd_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(
        static_cast<__nv_bfloat16*>(da), static_cast<__nv_bfloat16*>(db), static_cast<const __nv_bfloat16*>(dy),
        n / 4, accumulate);
  else
    residual_bwd_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(static_cast<float*>(da), static_cast<float*>(db),
                                                             static_cast<const float*>(dy), n / 4, accumulate);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_cast(void* out, llmk_dtype out_dtype, const void* in, llmk_dtype in_dtype, long long n, void* stream) {
  if (!out || !in || n < 0) return fail(LLMK_ERR_INVALID_ARG, "cast");
  if (n % 4 || !a16(out) || !a16(in)) return fail(LLMK_ERR_UNSUPPORTED, "cast: n % 4");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = grid_for(n / 4, 256);
  if (in_dtype == LLMK_F32 && out_dtype == LLMK_BF16)
    cast_kernel<<<g, 256, 0, s>>>(static_cast<__nv_bfloat16*>(out), static_cast<const float*>(in), n / 4);
  else if (in_dtype == LLMK_F32 && out_dtype == LLMK_F16)
    cast_kernel<<<g, 256, 0, s>>>(static_cast<__half*>(out), static_cast<const float*>(in), n / 4);
  else if (in_dtype == LLMK_F16 || out_dtype == LLMK_F16)
    return fail(LLMK_ERR_UNSUPPORTED, "cast: fp16 only as an fp32 -> fp16 cast");
  else if (in_dtype == LLMK_BF16 && out_dtype == LLMK_F32)
    cast_kernel<<<g, 256, 0, s>>>(static_cast<float*>(out), static_cast<const __nv_bfloat16*>(in), n / 4);
  else if (in_dtype == LLMK_F32)
    cast_kernel<<<g, 256, 0, s>>>(static_cast<float*>(out), static_cast<const float*>(in), n / 4);
  else
    cast_kernel<<<g, 256, 0, s>>>(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(in), n / 4);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_encoder_forward(float* out, const int* tokens, const float* wte, const float* wpe, int B, int T, int C,
                         void* stream) {
  if (!out || !tokens || !wte || !wpe || B <= 0 || T <= 0 || C <= 0) return fail(LLMK_ERR_INVALID_ARG, "encoder_forward");
  if (C % 4 || !a16(out) || !a16(wte) || !a16(wpe)) return fail(LLMK_ERR_UNSUPPORTED, "encoder_forward: C % 4");
  encoder_fwd_kernel<<<grid_for(static_cast<long long>(B) * T * C / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      out, tokens, wte, wpe, B * T, T, C);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

size_t llmk_encoder_backward_workspace(int B, int T) { return static_cast<size_t>(2) * B * T * sizeof(int); }

int llmk_encoder_backward(float* dwte, float* dwpe, const float* dout, const int* tokens, int B, int T, int C, int V,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!dwte || !dwpe || !dout || !tokens || B <= 0 || T <= 0 || C <= 0 || V <= 0)
    return fail(LLMK_ERR_INVALID_ARG, "encoder_backward");
  if (C % 4 || !a16(dwte) || !a16(dwpe) || !a16(dout)) return fail(LLMK_ERR_UNSUPPORTED, "encoder_backward: C % 4");
  if (!workspace || workspace_bytes < llmk_encoder_backward_workspace(B, T))
    return fail(LLMK_ERR_WORKSPACE, "encoder_backward: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int BT = B * T;
  encoder_bwd_wpe_kernel<<<grid_for(static_cast<long long>(T) * C / 4, 256), 256, 0, s>>>(dwpe, dout, B, T, C);
  if (BT <= kSortMaxBT && V < (1 << 17)) {
    // sort (token, position) keys once, then one pass over runs of equal tokens
    int n = 1;
    while (n < BT) n <<= 1;
    unsigned int* sorted = static_cast<unsigned int*>(workspace);
    if (BT <= kRadixMaxBT && V <= (1 << 16)) {
      LLMK_CUDA(cudaFuncSetAttribute(encoder_radix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kRadixSmem)));
      encoder_radix_kernel<<<1, 1024, kRadixSmem, s>>>(sorted, tokens, BT);
    } else if (n == 8192 || n == 16384) {  // (32 keys a thread would spill registers)
      const size_t smem = static_cast<size_t>(n + n / 32) * sizeof(unsigned int);
      auto kern = n == 8192 ? encoder_sort_reg_kernel<8> : encoder_sort_reg_kernel<16>;
      LLMK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      kern<<<1, 1024, smem, s>>>(sorted, tokens, BT);
    } else {
      const size_t smem = static_cast<size_t>(n) * sizeof(unsigned int);
      LLMK_CUDA(cudaFuncSetAttribute(encoder_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
      encoder_sort_kernel<<<1, 1024, smem, s>>>(sorted, tokens, BT, n);
    }
    // the list of long runs (a count, then their first sorted indices) in the
    // workspace's second half
    int* long_runs = static_cast<int*>(workspace) + BT;
    LLMK_CUDA(cudaMemsetAsync(long_runs, 0, sizeof(int), s));
    encoder_bwd_wte_sorted_kernel<<<grid_for(static_cast<long long>(BT) * C / 4, 256), 256, 0, s>>>(dwte, dout, sorted,
                                                                                                   BT, C, long_runs);
    encoder_bwd_wte_long_kernel<<<dim3(16, (C + 127) / 128), 1024, 0, s>>>(dwte, dout, sorted, BT, C, long_runs);
    count_launch(1);
  } else {
    int* first_of = static_cast<int*>(workspace);
    int* next_same = first_of + BT;
    encoder_links_kernel<<<(BT + 255) / 256, 256, 0, s>>>(first_of, next_same, tokens, BT);
    encoder_bwd_wte_kernel<<<grid_for(static_cast<long long>(BT) * C / 4, 256), 256, 0, s>>>(dwte, dout, tokens,
                                                                                            first_of, next_same, BT, C);
  }
  count_launch(3);
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_softmax_crossentropy(float* losses, void* dlogits, const void* logits, llmk_dtype dtype, const int* targets,
                              int BT, int V, int Vp, float dscale, void* stream) {
  if (!losses || !logits || !targets || BT <= 0 || V <= 0 || Vp < V)
    return fail(LLMK_ERR_INVALID_ARG, "softmax_crossentropy");
  if (Vp % 4 || !a16(logits) || !a16(dlogits)) return fail(LLMK_ERR_UNSUPPORTED, "softmax_crossentropy: Vp % 4");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LLMK_BF16)
    softmax_xent_kernel<__nv_bfloat16><<<BT, 512, 0, s>>>(losses, static_cast<__nv_bfloat16*>(dlogits),
                                                          static_cast<const __nv_bfloat16*>(logits), targets, V, Vp,
                                                          dscale);
  else
    softmax_xent_kernel<float><<<BT, 512, 0, s>>>(losses, static_cast<float*>(dlogits),
                                                  static_cast<const float*>(logits), targets, V, Vp, dscale);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_softmax_forward(void* probs, const void* logits, llmk_dtype dtype, int rows, int V, int ld, void* stream) {
  if (!probs || !logits || rows <= 0 || V <= 0 || ld < V) return fail(LLMK_ERR_INVALID_ARG, "softmax_forward");
  if (dtype != LLMK_F32 && dtype != LLMK_BF16) return fail(LLMK_ERR_UNSUPPORTED, "softmax_forward: fp32 or bf16");
  if (ld % 8 || !a16(logits) || !a16(probs)) return fail(LLMK_ERR_UNSUPPORTED, "softmax_forward: ld % 8, 16-byte rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LLMK_BF16)
    softmax_xent_kernel<__nv_bfloat16, true><<<rows, 512, 0, s>>>(
        nullptr, static_cast<__nv_bfloat16*>(probs), static_cast<const __nv_bfloat16*>(logits), nullptr, V, ld, 1.f);
  else
    softmax_xent_kernel<float, true><<<rows, 512, 0, s>>>(nullptr, static_cast<float*>(probs),
                                                          static_cast<const float*>(logits), nullptr, V, ld, 1.f);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_crossentropy_forward(float* losses, const void* probs, llmk_dtype dtype, const int* targets, int rows, int ld,
                              int accumulate, void* stream) {
  if (!losses || !probs || !targets || rows <= 0 || ld <= 0) return fail(LLMK_ERR_INVALID_ARG, "crossentropy_forward");
  if (dtype != LLMK_F32 && dtype != LLMK_BF16) return fail(LLMK_ERR_UNSUPPORTED, "crossentropy_forward: fp32 or bf16");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = (rows + 255) / 256;
  if (dtype == LLMK_BF16)
    xent_from_probs_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        losses, static_cast<const __nv_bfloat16*>(probs), targets, rows, ld, accumulate);
  else
    xent_from_probs_kernel<float><<<blocks, 256, 0, s>>>(losses, static_cast<const float*>(probs), targets, rows, ld,
                                                         accumulate);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_crossentropy_softmax_backward(void* dlogits, const void* probs, llmk_dtype dtype, const int* targets,
                                       int rows, int V, int ld, float scale, int accumulate, void* stream) {
  if (!dlogits || !probs || !targets || rows <= 0 || V <= 0 || ld < V)
    return fail(LLMK_ERR_INVALID_ARG, "crossentropy_softmax_backward");
  if (dtype != LLMK_F32 && dtype != LLMK_BF16)
    return fail(LLMK_ERR_UNSUPPORTED, "crossentropy_softmax_backward: fp32 or bf16");
  if (rows > 65535 * 1024) return fail(LLMK_ERR_UNSUPPORTED, "crossentropy_softmax_backward: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // rows on grid.y (chunks of 65535), columns on grid.x
  const int cx = std::min((V + 255) / 256, 16);
  for (int r0 = 0; r0 < rows; r0 += 65535) {
    const int n = std::min(65535, rows - r0);
    dim3 grid(cx, n);
    const size_t off = static_cast<size_t>(r0) * ld * (dtype == LLMK_BF16 ? 2 : 4);
    if (dtype == LLMK_BF16)
      xent_softmax_backward_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(dlogits) + off),
          reinterpret_cast<const __nv_bfloat16*>(static_cast<const char*>(probs) + off), targets + r0, V, ld, scale,
          accumulate);
    else
      xent_softmax_backward_kernel<float><<<grid, 256, 0, s>>>(
          reinterpret_cast<float*>(static_cast<char*>(dlogits) + off),
          reinterpret_cast<const float*>(static_cast<const char*>(probs) + off), targets + r0, V, ld, scale,
          accumulate);
    count_launch();
  }
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_mean(float* out, const float* x, int n, void* stream) {
  if (!out || !x || n <= 0) return fail(LLMK_ERR_INVALID_ARG, "mean");
  mean_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(out, x, n);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

int llmk_adamw(float* params, void* params_bf16, const float* grads, float* m, float* v, long long n, float lr,
               float beta1, float beta2, float eps, float weight_decay, int t, float grad_scale, void* stream) {
  if (!params || !grads || !m || !v || n < 0 || t < 1) return fail(LLMK_ERR_INVALID_ARG, "adamw");
  if (n % 4 || !a16(params) || !a16(params_bf16) || !a16(grads) || !a16(m) || !a16(v))
    return fail(LLMK_ERR_UNSUPPORTED, "adamw: n % 4 == 0 and 16-byte alignment required");
  // bias corrections in double on the host, as gpt2/cuda/adamw.cu:38-40
  const float inv_c1 = static_cast<float>(1.0 / (1.0 - std::pow(static_cast<double>(beta1), t)));
  const float inv_c2 = static_cast<float>(1.0 / (1.0 - std::pow(static_cast<double>(beta2), t)));
  const AdamHP hp{lr, beta1, beta2, eps, weight_decay, inv_c1, inv_c2, grad_scale};
  adamw_kernel<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      params, static_cast<__nv_bfloat16*>(params_bf16), grads, m, v, n / 4, hp, nullptr);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

void llmk_adamw_hparams(float* out8, float lr, float beta1, float beta2, float eps, float weight_decay, int t,
                        float grad_scale) {
  if (!out8) return;
  out8[0] = lr;
  out8[1] = beta1;
  out8[2] = beta2;
  out8[3] = eps;
  out8[4] = weight_decay;
  out8[5] = static_cast<float>(1.0 / (1.0 - std::pow(static_cast<double>(beta1), t > 0 ? t : 1)));
  out8[6] = static_cast<float>(1.0 / (1.0 - std::pow(static_cast<double>(beta2), t > 0 ? t : 1)));
  out8[7] = grad_scale;
}

int llmk_adamw_device_hparams(float* params, void* params_bf16, const float* grads, float* m, float* v, long long n,
                              const float* hparams, void* stream) {
  if (!params || !grads || !m || !v || n < 0 || !hparams) return fail(LLMK_ERR_INVALID_ARG, "adamw_device_hparams");
  if (n % 4 || !a16(params) || !a16(params_bf16) || !a16(grads) || !a16(m) || !a16(v) || !a16(hparams))
    return fail(LLMK_ERR_UNSUPPORTED, "adamw_device_hparams: n % 4 == 0 and 16-byte alignment required");
  adamw_kernel<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      params, static_cast<__nv_bfloat16*>(params_bf16), grads, m, v, n / 4, AdamHP{},
      reinterpret_cast<const AdamHP*>(hparams));
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

}  // extern "C"
