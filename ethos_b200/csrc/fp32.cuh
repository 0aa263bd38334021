// fp32 arithmetic path of the ETHOS expert layer (modules whose parameters
// are fp32; the reference then runs SimplifiedHypernetMoE / ProductKeyRouter,
// model.py:208-343, entirely in fp32).
//
// Contractions run on the tcgen05 GEMMs with split-bf16 operands: an fp32
// value v is carried as hi = bf16(v) and lo = bf16(v - hi) (16 significant
// bits together), and a product is formed as hi*hi + lo*hi + hi*lo with fp32
// accumulation, which leaves a relative error near 2^-16 per product.  The
// three partial products run as three accumulating GEMMs on separate hi / lo
// operand arrays.  The query projection is the exception: training-mode
// BatchNorm over a small batch amplifies an error in qpre by up to
// 1 / (2 sqrt(eps)) (two tokens normalise to +-1, and for a column where they
// nearly agree the result turns on their difference), so it carries a third
// part r = bf16(v - hi - lo) (v = hi + lo + r exactly for normal fp32 values)
// and forms the six products hi*r + r*hi + lo*lo + lo*hi + hi*lo + hi*hi
// as one GEMM whose operands are the segments concatenated along K, so that
// its epilogue sees the whole sum at once.  The order matters: the MMA's fp32
// accumulator loses about half an ulp of the running sum per K step (measured
// on the device: a relative error of 5.7e-6 over 192 steps of 16 with hi*hi
// first), so the small products accumulate first, while the sum is small, and
// hi*hi's D / 16 steps come last.
// Everything between the contractions -- BatchNorm, scores, top-k, softmax,
// the expert table, GELU, gathers and reductions -- stays in fp32 in the
// kernels below, which favour plain, coalesced fp32 row access over the bf16
// path's packed layouts.
#pragma once

#include <cuda_bf16.h>

#include "sm100.cuh"

namespace ethos {

// ------------------------------------------------------------- split --
// Parts of an fp32 value v: hi = bf16(v), lo = bf16(v - hi), r = bf16(v - hi
// - lo) (both differences exact in fp32).  dst segment s (s < nseg) of row r,
// column c is at dst[r * ldd + c + s * seg_off] and holds the part that bits
// 2s..2s+1 of `parts` select (0 hi, 1 lo, 2 r).  Separate hi / lo arrays of
// the source's shape: nseg 2, parts SPLIT_HI_LO, seg_off = rows * ldd;
// K-concatenated operand: seg_off = cols, ldd = nseg * cols.
constexpr int SPLIT_HI_LO = 1 << 2;
// The six-product projection operands, smallest products first:
// A = [hi | r | lo | lo | hi | hi], B = [r | hi | lo | hi | lo | hi].
constexpr int SPLIT6_A = (2 << 2) | (1 << 4) | (1 << 6);
constexpr int SPLIT6_B = 2 | (1 << 4) | (1 << 8);

__global__ void k_split_bf16(const float* __restrict__ src, int64_t rows, int cols, int64_t lds,
                             __nv_bfloat16* __restrict__ dst, int64_t ldd, int64_t seg_off, int nseg, int parts) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float v = src[r * lds + c];
    __nv_bfloat16 part[3];
    part[0] = __float2bfloat16_rn(v);
    const float rem = v - __bfloat162float(part[0]);
    part[1] = __float2bfloat16_rn(rem);
    part[2] = __float2bfloat16_rn(rem - __bfloat162float(part[1]));
    __nv_bfloat16* d = dst + r * ldd + c;
    for (int s = 0; s < nseg; ++s) d[s * seg_off] = part[(parts >> (2 * s)) & 3];
  }
}

// ------------------------------------------------------------ router --
// Normalised queries q^ = (qpre - center) * scale + beta per column into
// qhat [2][H][T][dq/2] (half p, head h).  center is the batch mean (training)
// or the running mean (eval), scale = gamma / sqrt(var + eps) (colp.x of
// k_bn_finalize / k_bn_eval_colp); the centred form keeps the subtraction
// exact where qpre and center agree to many bits (the folded qpre * scale +
// offset form loses those bits to the rounding of the offset).
__global__ void k_bn_apply_f32(const float* __restrict__ qpre, const float2* __restrict__ colp,
                               const float* __restrict__ center, const float* __restrict__ beta, int T, int H,
                               int dq, float* __restrict__ qhat) {
  const int C = H * dq;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  const int h = col / dq;
  const int e = col - h * dq;
  const int half = dq >> 1;
  const int p = e >= half ? 1 : 0;
  const int i = e - p * half;
  const float scale = colp[col].x, m = center[col], b = beta[col];
  float* base = qhat + static_cast<int64_t>(p * H + h) * T * half + i;
  for (int t = blockIdx.y; t < T; t += gridDim.y)
    base[static_cast<int64_t>(t) * half] = fmaf(qpre[static_cast<int64_t>(t) * C + col] - m, scale, b);
}

// Warp-wide arg-max of (value, index) pairs: the larger value wins, the
// smaller index among equal values.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

// The KSEL largest of n <= 32 * M values held M per lane (value j of lane l
// is element l + 32 j; absent elements are -inf), in descending order:
// out_v[r], out_i[r] for r < KSEL, the same on every lane.
template <int M, int KSEL>
__device__ __forceinline__ void warp_topk(float (&v)[M], float (&out_v)[KSEL], int (&out_i)[KSEL]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < KSEL; ++r) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < M; ++j) {
      const int idx = lane + 32 * j;
      if (v[j] > best || (v[j] == best && idx < bi)) {
        best = v[j];
        bi = idx;
      }
    }
    warp_argmax(best, bi);
    out_v[r] = best;
    out_i[r] = bi;
#pragma unroll
    for (int j = 0; j < M; ++j)
      if (lane + 32 * j == bi) v[j] = -INFINITY;
  }
}

// Product-key selection from dense fp32 scores (model.py:224-245): one warp
// per (token, head); scores [2][H*T][ldk] (row h*T + t, the first K columns
// used).  Top-k of each half, top-k of the k x k candidate sums (the same set
// as the reference's top-2k per half: if (i, j) is in the top k of the grid,
// so is every (i', j) with a larger first-half score), fp32 softmax, ids
// i1*K + i2.
template <int TOPK>
__global__ void __launch_bounds__(256) k_topk_f32(const float* __restrict__ scores, int64_t ldk, int T, int H,
                                                   int K, int32_t* __restrict__ ids, float* __restrict__ w) {
  constexpr int M = 16;  // K <= 512
  constexpr int G = (TOPK * TOPK + 31) / 32;
  const int lane = threadIdx.x & 31;
  const int64_t HT = static_cast<int64_t>(H) * T;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); item < HT;
       item += nw) {
    const int t = static_cast<int>(item / H), h = static_cast<int>(item - static_cast<int64_t>(t) * H);
    float sv[2][TOPK];
    int si[2][TOPK];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float* row = scores + (static_cast<int64_t>(p) * HT + static_cast<int64_t>(h) * T + t) * ldk;
      float v[M];
#pragma unroll
      for (int j = 0; j < M; ++j) v[j] = (lane + 32 * j < K) ? row[lane + 32 * j] : -INFINITY;
      warp_topk<M, TOPK>(v, sv[p], si[p]);
    }
    float g[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int c = lane + 32 * j;
      if (c < TOPK * TOPK) {
        // candidate c = (a, b): sv[0][a] + sv[1][b], read with compile-time
        // indices (a select chain keeps the lists in registers)
        const int a = c / TOPK, b = c - a * TOPK;
        float va = sv[0][0], vb = sv[1][0];
#pragma unroll
        for (int u = 1; u < TOPK; ++u) {
          va = (a == u) ? sv[0][u] : va;
          vb = (b == u) ? sv[1][u] : vb;
        }
        g[j] = va + vb;
      } else {
        g[j] = -INFINITY;
      }
    }
    float gv[TOPK];
    int gi[TOPK];
    warp_topk<G, TOPK>(g, gv, gi);
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < TOPK; ++r) sum += expf(gv[r] - gv[0]);
    if (lane < TOPK) {
      int my_c = gi[0];
      float my_g = gv[0];
#pragma unroll
      for (int r = 1; r < TOPK; ++r) {
        my_c = (lane == r) ? gi[r] : my_c;
        my_g = (lane == r) ? gv[r] : my_g;
      }
      const int a = my_c / TOPK, b = my_c - a * TOPK;
      int i1 = si[0][0], i2 = si[1][0];
#pragma unroll
      for (int u = 1; u < TOPK; ++u) {
        i1 = (a == u) ? si[0][u] : i1;
        i2 = (b == u) ? si[1][u] : i2;
      }
      const int64_t o = (static_cast<int64_t>(t) * H + h) * TOPK + lane;
      ids[o] = i1 * K + i2;
      w[o] = expf(my_g - gv[0]) / sum;
    }
  }
}

// ------------------------------------------------------------ experts --
// In place: tab[e][c] = gelu(pre) and, when g is given, g[e][c] = gelu'(pre)
// (the expert table of model.py:323, once per expert).
__global__ void k_gelu_table_f32(float* __restrict__ tab, float* __restrict__ g, int64_t n) {
  for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 2; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x * 2) {
    const float2 v = *reinterpret_cast<const float2*>(tab + i);
    float g0, g1, d0, d1;
    gelu_erf_and_grad2(v.x, v.y, g0, g1, d0, d1);
    *reinterpret_cast<float2*>(tab + i) = make_float2(g0, g1);
    if (g != nullptr) *reinterpret_cast<float2*>(g + i) = make_float2(d0, d1);
  }
}

// 512-wide fp32 rows, one warp per row: lane l owns columns 4l..4l+3 of each
// 128-column quarter q (float4 index l + 32 q).
__device__ __forceinline__ void load_row512(const float* row, float4 (&v)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = __ldg(reinterpret_cast<const float4*>(row) + lane + 32 * q);
}
__device__ __forceinline__ float dot_row512(const float4 (&a)[4], const float4 (&b)[4]) {
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    s = fmaf(a[q].x, b[q].x, s);
    s = fmaf(a[q].y, b[q].y, s);
    s = fmaf(a[q].z, b[q].z, s);
    s = fmaf(a[q].w, b[q].w, s);
  }
  return s;
}
__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}
__device__ __forceinline__ void axpy_row512(float a, const float4 (&x)[4], float4 (&y)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    y[q].x = fmaf(a, x[q].x, y[q].x);
    y[q].y = fmaf(a, x[q].y, y[q].y);
    y[q].z = fmaf(a, x[q].z, y[q].z);
    y[q].w = fmaf(a, x[q].w, y[q].w);
  }
}
__device__ __forceinline__ void store_row512(float* row, const float4 (&v)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < 4; ++q) reinterpret_cast<float4*>(row)[lane + 32 * q] = v[q];
}

// Per token t (one warp): dot_r = H[id_r] . xp_t, a_r = gelu(dot_r) w_r,
// hacc_t = sum_r a_r H[id_r] (model.py:320-338 in the reordered form).  Ids
// outside [0, N) read row 0 and set ETHOS_ERR_ID_OUT_OF_RANGE.
__global__ void __launch_bounds__(256) k_gather_f32(const float* __restrict__ table, const int32_t* __restrict__ ids,
                                                    const float* __restrict__ w, const float* __restrict__ xp,
                                                    float* __restrict__ hacc, float* __restrict__ dot_out, int T,
                                                    int R, int N, int* err) {
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  bool bad = false;
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += nw) {
    float4 xv[4], acc[4];
    load_row512(xp + static_cast<int64_t>(t) * 512, xv);
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < R; r0 += 4) {
      float4 hv[4][4];
      float part[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int id = __ldg(ids + static_cast<int64_t>(t) * R + r0 + u);
        if (static_cast<unsigned>(id) >= static_cast<unsigned>(N)) {
          bad = true;
          id = 0;
        }
        load_row512(table + static_cast<int64_t>(id) * 512, hv[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) part[u] = warp_sum(dot_row512(hv[u], xv));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float a = gelu_erf(part[u]) * __ldg(w + static_cast<int64_t>(t) * R + r0 + u);
        axpy_row512(a, hv[u], acc);
      }
      if (dot_out != nullptr && lane < 4) {
        float d = part[0];
#pragma unroll
        for (int u = 1; u < 4; ++u) d = lane == u ? part[u] : d;
        dot_out[static_cast<int64_t>(t) * R + r0 + lane] = d;
      }
    }
    store_row512(hacc + static_cast<int64_t>(t) * 512, acc);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
}

// ----------------------------------------------------------- backward --
// Per token t (one warp), for each selection r with h = H[id_r]:
//   da = dhacc_t . h,  dw_r = da gelu(dot_r),  a_r = gelu(dot_r) w_r,
//   ddot_r = da w_r gelu'(dot_r),  dxp_t = sum_r ddot_r h  (into du[t, off:])
__global__ void __launch_bounds__(256) k_bwd_token_f32(const float* __restrict__ table, const int32_t* __restrict__ ids,
                                                       const float* __restrict__ w, const float* __restrict__ dot,
                                                       const float* __restrict__ dhacc, float* __restrict__ dw_out,
                                                       float* __restrict__ ca_out, float* __restrict__ cd_out,
                                                       float* __restrict__ du, int64_t ldu, int du_off, int T, int R,
                                                       int N, int* err) {
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  bool bad = false;
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += nw) {
    float4 gv[4], acc[4];
    load_row512(dhacc + static_cast<int64_t>(t) * 512, gv);
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < R; r0 += 4) {
      float4 hv[4][4];
      float da[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int id = __ldg(ids + static_cast<int64_t>(t) * R + r0 + u);
        if (static_cast<unsigned>(id) >= static_cast<unsigned>(N)) {
          bad = true;
          id = 0;
        }
        load_row512(table + static_cast<int64_t>(id) * 512, hv[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) da[u] = warp_sum(dot_row512(hv[u], gv));
      float my_dw = 0.f, my_a = 0.f, my_dd = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t s = static_cast<int64_t>(t) * R + r0 + u;
        const float dt = __ldg(dot + s), wt = __ldg(w + s);
        const float gd = gelu_erf(dt), gp = gelu_erf_grad(dt);
        const float ddot = da[u] * wt * gp;
        axpy_row512(ddot, hv[u], acc);
        if (lane == u) {
          my_dw = da[u] * gd;
          my_a = gd * wt;
          my_dd = ddot;
        }
      }
      if (lane < 4) {
        const int64_t s = static_cast<int64_t>(t) * R + r0 + lane;
        dw_out[s] = my_dw;
        ca_out[s] = my_a;
        cd_out[s] = my_dd;
      }
    }
    store_row512(du + static_cast<int64_t>(t) * ldu + du_off, acc);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
}

// Per expert e (one warp): dP[e] = G[e] * sum_{s in seg(e)} (a_s dhacc_t +
// ddot_s xp_t), t = s / R, over the selections grouped by the counting sort
// (`total`: the device count of sorted selections); experts without
// selections get zeros.
__global__ void __launch_bounds__(256) k_expert_dP_f32(const int* __restrict__ offs, const int* __restrict__ perm,
                                                       const int* __restrict__ total, const float* __restrict__ ca,
                                                       const float* __restrict__ cd, const float* __restrict__ dhacc,
                                                       const float* __restrict__ xp, const float* __restrict__ gtab,
                                                       float* __restrict__ dP, int N, int R) {
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); e < N; e += nw) {
    const int s0 = offs[e], s1 = e + 1 < N ? offs[e + 1] : *total;
    float4 acc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = s0; k < s1; ++k) {
      const int s = __ldg(perm + k);
      const int t = s / R;
      float4 dv[4], xv[4];
      load_row512(dhacc + static_cast<int64_t>(t) * 512, dv);
      load_row512(xp + static_cast<int64_t>(t) * 512, xv);
      axpy_row512(__ldg(ca + s), dv, acc);
      axpy_row512(__ldg(cd + s), xv, acc);
    }
    float4 gv[4];
    load_row512(gtab + static_cast<int64_t>(e) * 512, gv);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[q].x *= gv[q].x;
      acc[q].y *= gv[q].y;
      acc[q].z *= gv[q].z;
      acc[q].w *= gv[q].w;
    }
    store_row512(dP + static_cast<int64_t>(e) * 512, acc);
  }
}

// Router backward per (token, head) (one warp; lane j < k holds selection j):
// softmax backward dg_j = w_j (dw_j - sum_i w_i dw_i) (model.py:234), the
// query-half gradients dq^_p = sum_j dg_j K_p[i_p,j] into dqhat [T, H*dq]
// (column h*dq + p*dq/2 + c), and the sub-key score gradient scattered into
// the dense dS [2][H*T][K] (zeroed by the caller) for the dK GEMMs.
template <int TOPK>
__global__ void __launch_bounds__(256) k_router_bwd_f32(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                        const float* __restrict__ dw, const float* __restrict__ keys,
                                                        float* __restrict__ dqhat, float* __restrict__ dS, int T,
                                                        int H, int K, int dq) {
  const int lane = threadIdx.x & 31;
  const int half = dq >> 1;
  const int64_t HT = static_cast<int64_t>(H) * T;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); item < HT;
       item += nw) {
    const int t = static_cast<int>(item / H), h = static_cast<int>(item - static_cast<int64_t>(t) * H);
    const int64_t o = (static_cast<int64_t>(t) * H + h) * TOPK;
    float wj = 0.f, dwj = 0.f;
    int id = 0;
    // an id outside [0, K*K) (reported by k_count_experts) contributes nothing
    if (lane < TOPK && static_cast<unsigned>(ids[o + lane]) < static_cast<unsigned>(K * K)) {
      wj = w[o + lane];
      dwj = dw[o + lane];
      id = ids[o + lane];
    }
    const float s = warp_sum(wj * dwj);
    const float dg = lane < TOPK ? wj * (dwj - s) : 0.f;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int idx = p == 0 ? id / K : id - (id / K) * K;
      if (lane < TOPK && dg != 0.f)
        atomicAdd(dS + (static_cast<int64_t>(p) * HT + static_cast<int64_t>(h) * T + t) * K + idx, dg);
      const float* kp = keys + static_cast<int64_t>(p) * K * half;
      float* out = dqhat + static_cast<int64_t>(t) * H * dq + h * dq + p * half;
      for (int c = lane; c < half; c += 32) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < TOPK; ++j) {
          const float g = __shfl_sync(0xffffffffu, dg, j);
          const int ij = __shfl_sync(0xffffffffu, idx, j);
          acc = fmaf(g, kp[static_cast<int64_t>(ij) * half + c], acc);
        }
        out[c] = acc;
      }
    }
  }
}

// BatchNorm backward apply (k_bn_bwd_apply with an fp32 destination):
// du[t][c] = A dq^ + B (qpre - mean) + D per column, coef[c] = (A, B, D, mean).
__global__ void k_bn_bwd_apply_f32(const float* __restrict__ dqh, const float* __restrict__ qpre,
                                   const float4* __restrict__ coef, int T, int C, float* __restrict__ du,
                                   int64_t ldu) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float4 k = __ldg(coef + c);
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const int64_t o = static_cast<int64_t>(t) * C + c;
    du[static_cast<int64_t>(t) * ldu + c] = fmaf(k.x, dqh[o], fmaf(k.y, qpre[o] - k.w, k.z));
  }
}

}  // namespace ethos
