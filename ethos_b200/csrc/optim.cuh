// Fused multi-tensor AdamW (torch.optim.AdamW semantics, decoupled weight
// decay, bias correction), one launch for all of a layer's parameters.
// Grid: y = tensor, x = element blocks walked with a grid stride; 4 elements
// per thread and iteration (float4 / 2 x bf16x2 accesses when the tensor's
// buffers are 16-byte aligned and n % 4 == 0, scalar otherwise).  HBM-bound:
// per element 4 B grad (2 bf16) + 2 x 8 B moments + 8 B master + 2-4 B param.
#pragma once

#include <cuda_bf16.h>

#include "ethos_b200.h"

namespace ethos {

struct AdamScalars {
  float lr, beta1, beta2, eps, wd;
  float step_size;  // lr / (1 - beta1^step)
  float bc2_sqrt;   // sqrt(1 - beta2^step)
};

__device__ __forceinline__ float adam_elem(float p, float g, float& m, float& v, const AdamScalars& s) {
  p = p * (1.0f - s.lr * s.wd);
  m = fmaf(1.0f - s.beta1, g - m, m);            // lerp(m, g, 1 - beta1)
  v = fmaf(1.0f - s.beta2, g * g, s.beta2 * v);  // v * beta2 + (1 - beta2) g^2
  const float denom = sqrtf(v) / s.bc2_sqrt + s.eps;
  return p - s.step_size * (m / denom);
}

// grad_scale (device, may be null): every gradient is multiplied by
// grad_scale[0] before the update (the clip coefficient of k_grad_clip_coef)
__global__ void k_adamw(const ethos_adam_tensor* __restrict__ tensors, AdamScalars s,
                        const float* __restrict__ grad_scale) {
  const ethos_adam_tensor td = tensors[blockIdx.y];
  const float gs = grad_scale != nullptr ? *grad_scale : 1.0f;
  const int64_t n = td.n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(td.param) | reinterpret_cast<uintptr_t>(td.grad) |
                                     reinterpret_cast<uintptr_t>(td.exp_avg) |
                                     reinterpret_cast<uintptr_t>(td.exp_avg_sq) |
                                     reinterpret_cast<uintptr_t>(td.master)) & 15u) == 0 &&
                   (!td.param_bf16 || (reinterpret_cast<uintptr_t>(td.param) & 7u) == 0);
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    float g[4], p[4], m[4], v[4];
    const int cnt = static_cast<int>(n - i < 4 ? n - i : 4);
    if (vec) {
      if (td.grad_bf16) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(td.grad) + i);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        g[0] = a.x; g[1] = a.y; g[2] = b.x; g[3] = b.y;
      } else {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(td.grad) + i);
        g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w;
      }
      const float4 ma = *reinterpret_cast<const float4*>(td.exp_avg + i);
      const float4 va = *reinterpret_cast<const float4*>(td.exp_avg_sq + i);
      m[0] = ma.x; m[1] = ma.y; m[2] = ma.z; m[3] = ma.w;
      v[0] = va.x; v[1] = va.y; v[2] = va.z; v[3] = va.w;
      if (td.master != nullptr) {
        const float4 pa = *reinterpret_cast<const float4*>(td.master + i);
        p[0] = pa.x; p[1] = pa.y; p[2] = pa.z; p[3] = pa.w;
      } else if (td.param_bf16) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(td.param) + i);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        p[0] = a.x; p[1] = a.y; p[2] = b.x; p[3] = b.y;
      } else {
        const float4 pa = *reinterpret_cast<const float4*>(static_cast<const float*>(td.param) + i);
        p[0] = pa.x; p[1] = pa.y; p[2] = pa.z; p[3] = pa.w;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) p[u] = adam_elem(p[u], g[u] * gs, m[u], v[u], s);
      *reinterpret_cast<float4*>(td.exp_avg + i) = make_float4(m[0], m[1], m[2], m[3]);
      *reinterpret_cast<float4*>(td.exp_avg_sq + i) = make_float4(v[0], v[1], v[2], v[3]);
      if (td.master != nullptr) *reinterpret_cast<float4*>(td.master + i) = make_float4(p[0], p[1], p[2], p[3]);
      if (td.param_bf16) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(p[0], p[1]), b = __floats2bfloat162_rn(p[2], p[3]);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&a);
        u.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(td.param) + i) = u;
      } else {
        *reinterpret_cast<float4*>(static_cast<float*>(td.param) + i) = make_float4(p[0], p[1], p[2], p[3]);
      }
    } else {
      for (int u = 0; u < cnt; ++u) {
        const int64_t j = i + u;
        const float gg = (td.grad_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(td.grad)[j])
                                       : static_cast<const float*>(td.grad)[j]) *
                         gs;
        float mm = td.exp_avg[j], vv = td.exp_avg_sq[j];
        const float pp = td.master != nullptr ? td.master[j]
                         : td.param_bf16      ? __bfloat162float(static_cast<const __nv_bfloat16*>(td.param)[j])
                                              : static_cast<const float*>(td.param)[j];
        const float np = adam_elem(pp, gg, mm, vv, s);
        td.exp_avg[j] = mm;
        td.exp_avg_sq[j] = vv;
        if (td.master != nullptr) td.master[j] = np;
        if (td.param_bf16)
          static_cast<__nv_bfloat16*>(td.param)[j] = __float2bfloat16_rn(np);
        else
          static_cast<float*>(td.param)[j] = np;
      }
    }
  }
}

// ---------------------------------------------------- gradient clipping --
// Global-norm clipping as torch.nn.utils.clip_grad_norm_ (and DeepSpeed's
// gradient_clipping, train.py:100) defines it: norm = sqrt(sum of every
// gradient element squared), coef = min(1, max_norm / (norm + 1e-6)).  The sum
// does not depend on scheduling, so data-parallel ranks holding the same
// all-reduced gradients get bit-identical coefficients: a fixed grid of
// GRAD_CLIP_BLOCKS blocks walks every tensor in table order, each thread
// taking fixed chunks of each and accumulating in fp64; block b writes its
// sum to partial[b], and one block adds the partials in a fixed order.
constexpr int GRAD_CLIP_BLOCKS = 1184;  // 8 per SM of a B200; fixed, so the sum's order is too
constexpr int GRAD_CLIP_THREADS = 256;

// sum of squares of 8 gradient elements (16 bytes of bf16 or 32 of fp32)
__device__ __forceinline__ double sq8(const ethos_adam_tensor& td, int64_t c) {
  float g[8];
  if (td.grad_bf16) {
    const uint4 u = *(reinterpret_cast<const uint4*>(td.grad) + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      g[2 * k] = f.x;
      g[2 * k + 1] = f.y;
    }
  } else {
    const float4 a = *(reinterpret_cast<const float4*>(td.grad) + 2 * c);
    const float4 b = *(reinterpret_cast<const float4*>(td.grad) + 2 * c + 1);
    g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w; g[4] = b.x; g[5] = b.y; g[6] = b.z; g[7] = b.w;
  }
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < 8; ++k) s = fma(static_cast<double>(g[k]), static_cast<double>(g[k]), s);
  return s;
}

// Thread t takes the 8-element chunks t, t + T, t + 2T, ... (T = threads of
// the grid) of every tensor, two chunks' loads in flight at a time; a tensor
// whose size or address does not allow 16-byte chunks is walked element by
// element instead.  The assignment depends only on the sizes.
__global__ void __launch_bounds__(GRAD_CLIP_THREADS) k_grad_sqnorm(const ethos_adam_tensor* __restrict__ tensors,
                                                                   int num_tensors, double* __restrict__ partial) {
  __shared__ double red[GRAD_CLIP_THREADS];
  const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  double acc = 0.0;
  for (int y = 0; y < num_tensors; ++y) {
    const ethos_adam_tensor td = tensors[y];
    const int64_t n = td.n;
    if (n % 8 == 0 && (reinterpret_cast<uintptr_t>(td.grad) & 15u) == 0) {
      const int64_t nc = n / 8;
      int64_t c = tid;
      for (; c + nt < nc; c += 2 * nt) {
        const double a = sq8(td, c), b = sq8(td, c + nt);
        acc += a;
        acc += b;
      }
      if (c < nc) acc += sq8(td, c);
    } else {
      for (int64_t j = tid; j < n; j += nt) {
        const float g = td.grad_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(td.grad)[j])
                                     : static_cast<const float*>(td.grad)[j];
        acc = fma(static_cast<double>(g), static_cast<double>(g), acc);
      }
    }
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = GRAD_CLIP_THREADS / 2; w > 0; w >>= 1) {
    if (static_cast<int>(threadIdx.x) < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

// out[0] = norm, out[1] = min(1, max_norm / (norm + 1e-6)); one block
__global__ void __launch_bounds__(GRAD_CLIP_THREADS) k_grad_clip_coef(const double* __restrict__ partial, int count,
                                                                      float max_norm, float* __restrict__ out) {
  __shared__ double red[GRAD_CLIP_THREADS];
  double acc = 0.0;
  for (int i = threadIdx.x; i < count; i += blockDim.x) acc += partial[i];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = GRAD_CLIP_THREADS / 2; w > 0; w >>= 1) {
    if (static_cast<int>(threadIdx.x) < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float norm = static_cast<float>(sqrt(red[0]));
    const float coef = max_norm / (norm + 1e-6f);
    out[0] = norm;
    out[1] = coef > 1.0f ? 1.0f : coef;  // a NaN norm stays NaN, as torch.clamp leaves it
  }
}

}  // namespace ethos
