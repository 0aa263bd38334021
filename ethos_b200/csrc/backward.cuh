// Backward pass of the ETHOS expert layer.
//
// Reference: autograd through SimplifiedHypernetMoE.forward (model.py:288-343)
// and ProductKeyRouter.forward (model.py:208-254).  With a_r = gelu(dot_r) w_r,
// h_r = gelu(pre_r), pre_r = E[id_r] W1^T, dot_r = h_r . xp_t:
//   dhacc_t = dy_t W_v / H                         (GEMM)
//   da_r    = dhacc_t . h_r
//   dw_r    = da_r gelu(dot_r)                     (routing-weight gradient)
//   ddot_r  = da_r w_r gelu'(dot_r)
//   dxp_t   = sum_r ddot_r h_r
//   dh_r    = a_r dhacc_t + ddot_r xp_t
//   dpre_r  = dh_r * gelu'(pre_r)
// Because pre_r depends only on the expert e = id_r, the expert-side
// gradients aggregate per expert: dP[e] = gelu'(P[e]) * sum_{r: id_r = e} dh_r,
// after which dE = dP W1 and dW1 = dP^T E are dense GEMMs.  The selections
// are grouped by expert with a counting sort; dhacc and xp (64 MB at the
// default size) stay L2-resident while each expert sums its selections.
#pragma once

#include <cuda_fp16.h>

#include "expert_table.cuh"
#include "router.cuh"

namespace ethos {

// ------------------------------------------------------------------------
// Per-token backward gather: the forward gather kernel's structure with the
// token vector dhacc in place of xp.  Per selection it writes dw, a and ddot;
// per token dxp (fp32) and its bf16 copy into the GEMM operand du[:, off:].
// Warps per block, cp.async ring depth and per-token buffers.  A token's
// dhacc / xp vectors move to registers at its first batch and the next
// token's copies are issued STAGES-1 batches ahead, so one buffer each is
// enough while STAGES-1 < batches per token (R / 4); for R = 4 the host
// launches a double-buffered instance (safe while STAGES-1 < 2 R / 4).
// (B200, 16384 tokens x 128 selections, whole backward: 8x5 2.68 ms,
// 10x3 2.65, 12x2 2.55 with double buffers; 16x2 single-buffered below)
#ifndef ETHOS_BGATHER_WARPS
#define ETHOS_BGATHER_WARPS 16
#endif
#ifndef ETHOS_BGATHER_STAGES
#define ETHOS_BGATHER_STAGES 2
#endif
constexpr int BGATHER_WARPS = ETHOS_BGATHER_WARPS;
constexpr int BGATHER_STAGES = ETHOS_BGATHER_STAGES;
constexpr int BGATHER_SMALL_R_WARPS = 12;  // the double-buffered instance
constexpr int BGATHER_STAGE_BYTES = GATHER_ROWS * 1024 + 32;  // rows + 4 weights + 4 dots
// + per-token buffers for dhacc and xp (fp32, 2 KB each), nbuf deep
__host__ __device__ constexpr int bgather_warp_bytes(int stages, int nbuf) {
  return stages * BGATHER_STAGE_BYTES + nbuf * 2048 + nbuf * 2048;
}
__host__ __device__ constexpr int bgather_smem_bytes(int warps, int stages, int nbuf) {
  return warps * bgather_warp_bytes(stages, nbuf);
}
static_assert(BGATHER_STAGES >= 2, "ring needs two stages");
static_assert(bgather_smem_bytes(BGATHER_WARPS, BGATHER_STAGES, 1) <= 227 * 1024,
              "backward gather ring exceeds shared memory");
static_assert(bgather_smem_bytes(BGATHER_SMALL_R_WARPS, 2, 2) <= 227 * 1024,
              "backward gather ring exceeds shared memory");

template <int WARPS, int STAGES, int NBUF>
__global__ void __launch_bounds__(WARPS * 32, 1)
    k_expert_bwd_gather(const __half* __restrict__ table, const int32_t* __restrict__ ids,
                        const float* __restrict__ w, const float* __restrict__ dot, const float* __restrict__ dhacc,
                        float* __restrict__ dw_out, float* __restrict__ ca_out, float* __restrict__ cd_out,
                        float* __restrict__ dxp_out, __nv_bfloat16* __restrict__ du, int64_t ldu, int du_off,
                        const float* __restrict__ xp, __nv_bfloat16* __restrict__ gx, int T, int R, int N, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  uint8_t* wbase = smem_raw + wib * bgather_warp_bytes(STAGES, NBUF);
  uint8_t* vbuf = wbase + STAGES * BGATHER_STAGE_BYTES;
  uint8_t* xbuf = vbuf + NBUF * 2048;
  const int gw = blockIdx.x * WARPS + wib;
  const int nw = gridDim.x * WARPS;
  const int nbt = R / GATHER_ROWS;
  const int ntok = T > gw ? (T - 1 - gw) / nw + 1 : 0;
  const int nb = ntok * nbt;
  const int b3 = (lane >> 3) & 1, b4 = (lane >> 4) & 1;
  const int grp = (lane >> 3) & 3;

  // Cursors instead of div/mod by the runtime batch count: the issue cursor
  // (token it_t, its local index it_k, row it_r) runs STAGES-1 batches ahead
  // of the consume cursor; the token index parity picks the dhacc / xp
  // double buffer.
  int it_t = gw, it_k = 0, it_r = 0, it_n = 0;
  bool bad_id = false;
  int4 next_ids = nb > 0 ? __ldg(reinterpret_cast<const int4*>(ids + static_cast<int64_t>(gw) * R))
                         : make_int4(0, 0, 0, 0);
  auto issue_next = [&]() {
    if (it_n < nb) {
      const int t = it_t, r0 = it_r;
      uint8_t* st = wbase + (it_n % STAGES) * BGATHER_STAGE_BYTES;
      const int idv[4] = {next_ids.x, next_ids.y, next_ids.z, next_ids.w};
#pragma unroll
      for (int u = 0; u < GATHER_ROWS; ++u) {
        const bool bad = static_cast<unsigned>(idv[u]) >= static_cast<unsigned>(N);
        bad_id |= bad;
        const char* src = reinterpret_cast<const char*>(table + static_cast<int64_t>(bad ? 0 : idv[u]) * 512);
        cp_async_16(st + u * 1024 + 16 * lane, src + 16 * lane);
        cp_async_16(st + u * 1024 + 512 + 16 * lane, src + 512 + 16 * lane);
      }
      if (lane == 0) cp_async_16(st + GATHER_ROWS * 1024, w + static_cast<int64_t>(t) * R + r0);
      if (lane == 1) cp_async_16(st + GATHER_ROWS * 1024 + 16, dot + static_cast<int64_t>(t) * R + r0);
      if (r0 == 0) {
        const char* xs = reinterpret_cast<const char*>(dhacc + static_cast<int64_t>(t) * 512);
        uint8_t* xd = vbuf + (it_k % NBUF) * 2048;
        cp_async_16(xd + 32 * lane, xs + 32 * lane);
        cp_async_16(xd + 32 * lane + 16, xs + 32 * lane + 16);
        cp_async_16(xd + 1024 + 32 * lane, xs + 1024 + 32 * lane);
        cp_async_16(xd + 1024 + 32 * lane + 16, xs + 1024 + 32 * lane + 16);
        const char* ps = reinterpret_cast<const char*>(xp + static_cast<int64_t>(t) * 512);
        uint8_t* pd = xbuf + (it_k % NBUF) * 2048;
        cp_async_16(pd + 32 * lane, ps + 32 * lane);
        cp_async_16(pd + 32 * lane + 16, ps + 32 * lane + 16);
        cp_async_16(pd + 1024 + 32 * lane, ps + 1024 + 32 * lane);
        cp_async_16(pd + 1024 + 32 * lane + 16, ps + 1024 + 32 * lane + 16);
      }
      ++it_n;
      it_r += GATHER_ROWS;
      if (it_r == R) {
        it_r = 0;
        it_t += nw;
        ++it_k;
      }
      if (it_n < nb) next_ids = __ldg(reinterpret_cast<const int4*>(ids + static_cast<int64_t>(it_t) * R + it_r));
    }
    cp_async_commit();
  };

#pragma unroll 1
  for (int b = 0; b < STAGES - 1; ++b) issue_next();
  float gv[16];
  unsigned long long gv2[8];   // dhacc columns as packed pairs
  unsigned long long acc2[8];  // dxp columns as packed pairs
#pragma unroll
  for (int i = 0; i < 8; ++i) acc2[i] = 0ull;
  int t = gw, tk = 0, r0 = 0;  // consume cursor
#pragma unroll 1
  for (int b = 0; b < nb; ++b) {
    issue_next();
    cp_async_wait_group<STAGES - 1>();
    const uint8_t* st = wbase + (b % STAGES) * BGATHER_STAGE_BYTES;
    if (r0 == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(vbuf + (tk % NBUF) * 2048);
      const float4 a0 = x4[2 * lane], a1 = x4[2 * lane + 1], c0 = x4[64 + 2 * lane], c1 = x4[64 + 2 * lane + 1];
      gv[0] = a0.x; gv[1] = a0.y; gv[2] = a0.z; gv[3] = a0.w;
      gv[4] = a1.x; gv[5] = a1.y; gv[6] = a1.z; gv[7] = a1.w;
      gv[8] = c0.x; gv[9] = c0.y; gv[10] = c0.z; gv[11] = c0.w;
      gv[12] = c1.x; gv[13] = c1.y; gv[14] = c1.z; gv[15] = c1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        gv2[i] = pk2(gv[2 * i], gv[2 * i + 1]);
        acc2[i] = 0ull;
      }
      // bf16 copy of this token's [dhacc | xp] row for the per-expert pass
      const float4* p4 = reinterpret_cast<const float4*>(xbuf + (tk % NBUF) * 2048);
      const float4 e0 = p4[2 * lane], e1 = p4[2 * lane + 1], f0 = p4[64 + 2 * lane], f1 = p4[64 + 2 * lane + 1];
      __nv_bfloat16* gr = gx + static_cast<int64_t>(t) * 1024;
      auto pk = [](float a, float b) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&v);
      };
      *reinterpret_cast<uint4*>(gr + 8 * lane) = make_uint4(pk(gv[0], gv[1]), pk(gv[2], gv[3]), pk(gv[4], gv[5]),
                                                            pk(gv[6], gv[7]));
      *reinterpret_cast<uint4*>(gr + 256 + 8 * lane) = make_uint4(pk(gv[8], gv[9]), pk(gv[10], gv[11]),
                                                                  pk(gv[12], gv[13]), pk(gv[14], gv[15]));
      *reinterpret_cast<uint4*>(gr + 512 + 8 * lane) = make_uint4(pk(e0.x, e0.y), pk(e0.z, e0.w), pk(e1.x, e1.y),
                                                                  pk(e1.z, e1.w));
      *reinterpret_cast<uint4*>(gr + 768 + 8 * lane) = make_uint4(pk(f0.x, f0.y), pk(f0.z, f0.w), pk(f1.x, f1.y),
                                                                  pk(f1.z, f1.w));
    }
    unsigned long long hf[GATHER_ROWS][8];
    float part[GATHER_ROWS];
#pragma unroll
    for (int u = 0; u < GATHER_ROWS; ++u) {
      unpack_h8_x2(*reinterpret_cast<const uint4*>(st + u * 1024 + 16 * lane), hf[u]);
      unpack_h8_x2(*reinterpret_cast<const uint4*>(st + u * 1024 + 512 + 16 * lane), hf[u] + 4);
      unsigned long long s2 = 0ull;
#pragma unroll
      for (int i = 0; i < 8; ++i) s2 = ffma2(hf[u][i], gv2[i], s2);
      float lo, hi;
      upk2(s2, lo, hi);
      part[u] = lo + hi;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = b4 ? part[i] : part[i + 2];
      const float keep = b4 ? part[i + 2] : part[i];
      part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    {
      const float send = b3 ? part[0] : part[1];
      const float keep = b3 ? part[1] : part[0];
      part[0] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float da = part[0] + __shfl_xor_sync(0xffffffffu, part[0], 4);
    da += __shfl_xor_sync(0xffffffffu, da, 2);
    da += __shfl_xor_sync(0xffffffffu, da, 1);
    const float wgt = reinterpret_cast<const float*>(st + GATHER_ROWS * 1024)[grp];
    const float dt = reinterpret_cast<const float*>(st + GATHER_ROWS * 1024 + 16)[grp];
    const float gd = gelu_erf(dt);
    const float ddot = da * wgt * gelu_erf_grad(dt);
    if ((lane & 7) == 0) {
      const int64_t o = static_cast<int64_t>(t) * R + r0 + grp;
      dw_out[o] = da * gd;
      ca_out[o] = gd * wgt;
      cd_out[o] = ddot;
    }
#pragma unroll
    for (int u = 0; u < GATHER_ROWS; ++u) {
      const float c = __shfl_sync(0xffffffffu, ddot, 8 * u);
      const unsigned long long c2 = pk2(c, c);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc2[i] = ffma2(c2, hf[u][i], acc2[i]);
    }
    if (r0 + GATHER_ROWS == R) {
      float acc[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) upk2(acc2[i], acc[2 * i], acc[2 * i + 1]);
      float* dst = dxp_out + static_cast<int64_t>(t) * 512;
      *reinterpret_cast<float4*>(dst + 8 * lane) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(dst + 8 * lane + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
      *reinterpret_cast<float4*>(dst + 256 + 8 * lane) = make_float4(acc[8], acc[9], acc[10], acc[11]);
      *reinterpret_cast<float4*>(dst + 256 + 8 * lane + 4) = make_float4(acc[12], acc[13], acc[14], acc[15]);
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162 bb = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      __nv_bfloat16* ud = du + static_cast<int64_t>(t) * ldu + du_off;
      *reinterpret_cast<uint4*>(ud + 8 * lane) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(ud + 256 + 8 * lane) = make_uint4(o[4], o[5], o[6], o[7]);
    }
    r0 += GATHER_ROWS;
    if (r0 == R) {
      r0 = 0;
      t += nw;
      ++tk;
    }
  }
  cp_async_wait_group<0>();
  if (__any_sync(0xffffffffu, bad_id) && lane == 0) record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
}

// ------------------------------------------------------------------------
// Counting sort of the T*R selections by expert id.
__global__ void k_count_experts(const int32_t* __restrict__ ids, int64_t n, int N, int* __restrict__ cnt, int* err) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[i];
    if (e < 0 || e >= N) {
      record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
      continue;
    }
    atomicAdd(cnt + e, 1);
  }
}

// Exclusive scan in three steps: per-block scan of 1024 counts (block sums
// out), scan of the block sums (one block), add-back.
__global__ void k_scan_blocks(const int* __restrict__ in, int n, int* __restrict__ out, int* __restrict__ sums) {
  __shared__ int s[1024];
  const int i = blockIdx.x * 1024 + threadIdx.x;
  const int v = i < n ? in[i] : 0;
  s[threadIdx.x] = v;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int add = threadIdx.x >= off ? s[threadIdx.x - off] : 0;
    __syncthreads();
    s[threadIdx.x] += add;
    __syncthreads();
  }
  if (i < n) out[i] = s[threadIdx.x] - v;
  if (threadIdx.x == 1023) sums[blockIdx.x] = s[1023];
}
__global__ void k_scan_sums(int* __restrict__ sums, int nblocks, int* __restrict__ total_out) {
  __shared__ int s[1024];
  const int v = threadIdx.x < nblocks ? sums[threadIdx.x] : 0;
  s[threadIdx.x] = v;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int add = threadIdx.x >= off ? s[threadIdx.x - off] : 0;
    __syncthreads();
    s[threadIdx.x] += add;
    __syncthreads();
  }
  if (threadIdx.x < nblocks) sums[threadIdx.x] = s[threadIdx.x] - v;
  if (threadIdx.x == 1023) *total_out = s[1023];
}
__global__ void k_scan_add(int* __restrict__ out, int n, const int* __restrict__ sums, int* __restrict__ cursor) {
  const int i = blockIdx.x * 1024 + threadIdx.x;
  if (i < n) {
    const int v = out[i] + sums[blockIdx.x];
    out[i] = v;
    cursor[i] = v;
  }
}
__global__ void k_scatter_experts(const int32_t* __restrict__ ids, int64_t n, int N, int* __restrict__ cursor,
                                  int* __restrict__ perm) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[i];
    if (e < 0 || e >= N) continue;
    const int pos = atomicAdd(cursor + e, 1);
    perm[pos] = static_cast<int>(i);
  }
}

// ------------------------------------------------------------------------
__device__ __forceinline__ void unpack_b8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

// Per-expert pre-activation gradient (one warp per expert, lane l owns hidden
// columns [8l, 8l+8) and [256+8l, 256+8l+8)):
//   dP[e] = G[e] * sum_{s in seg(e)} (a_s dhacc[t_s] + ddot_s xp[t_s])
// reading the bf16 token rows gx[t] = [dhacc | xp] (2 KB each, L2-resident)
// and writing bf16 (operand of the dE / dW1 GEMMs).  Experts without
// selections get zeros.  `total` is the device count of sorted selections
// (k_scan_sums), so segments never reach past the entries k_scatter_experts
// wrote.
__global__ void __launch_bounds__(256, 3) k_expert_dP(const int* __restrict__ offs, const int* __restrict__ perm,
                                                    const int* __restrict__ total, const float* __restrict__ ca,
                                                    const float* __restrict__ cd, const __nv_bfloat16* __restrict__ gx,
                                                    const __half* __restrict__ gtab, __nv_bfloat16* __restrict__ dP,
                                                    int N, int R) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int e = gw; e < N; e += nw) {
    const int s0 = offs[e];
    const int s1 = e + 1 < N ? offs[e + 1] : *total;  // selections with a valid id
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    for (int base = s0; base < s1; base += 32) {
      // lanes fetch up to 32 entries of the segment at once
      const int n = min(32, s1 - base);
      int my_t = 0;
      float my_a = 0.f, my_d = 0.f;
      if (lane < n) {
        const int idx = __ldg(perm + base + lane);
        my_t = idx / R;
        my_a = __ldg(ca + idx);
        my_d = __ldg(cd + idx);
      }
      for (int u0 = 0; u0 < n; u0 += 2) {
        uint4 rv[2][4];
        float av[2], dv[2];
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          const int u = u0 + v;
          const int t = __shfl_sync(0xffffffffu, my_t, u & 31);
          av[v] = __shfl_sync(0xffffffffu, my_a, u & 31);
          dv[v] = __shfl_sync(0xffffffffu, my_d, u & 31);
          if (u < n) {
            const __nv_bfloat16* row = gx + static_cast<int64_t>(t) * 1024;
            rv[v][0] = __ldg(reinterpret_cast<const uint4*>(row + 8 * lane));
            rv[v][1] = __ldg(reinterpret_cast<const uint4*>(row + 256 + 8 * lane));
            rv[v][2] = __ldg(reinterpret_cast<const uint4*>(row + 512 + 8 * lane));
            rv[v][3] = __ldg(reinterpret_cast<const uint4*>(row + 768 + 8 * lane));
          } else {
            av[v] = 0.f;
            dv[v] = 0.f;
            rv[v][0] = rv[v][1] = rv[v][2] = rv[v][3] = make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          float g0[8], g1[8], x0[8], x1[8];
          unpack_b8(rv[v][0], g0);
          unpack_b8(rv[v][1], g1);
          unpack_b8(rv[v][2], x0);
          unpack_b8(rv[v][3], x1);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc[i] = fmaf(av[v], g0[i], fmaf(dv[v], x0[i], acc[i]));
            acc[8 + i] = fmaf(av[v], g1[i], fmaf(dv[v], x1[i], acc[8 + i]));
          }
        }
      }
    }
    const __half* gr = gtab + static_cast<int64_t>(e) * 512;
    float gf[16];
    {
      float f[8];
      unpack_h8(*reinterpret_cast<const uint4*>(gr + 8 * lane), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) gf[i] = f[i];
      unpack_h8(*reinterpret_cast<const uint4*>(gr + 256 + 8 * lane), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) gf[8 + i] = f[i];
    }
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __nv_bfloat162 bb = __floats2bfloat162_rn(acc[2 * i] * gf[2 * i], acc[2 * i + 1] * gf[2 * i + 1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&bb);
    }
    __nv_bfloat16* dst = dP + static_cast<int64_t>(e) * 512;
    *reinterpret_cast<uint4*>(dst + 8 * lane) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(dst + 256 + 8 * lane) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// ------------------------------------------------------------------------
// Router backward per (token, head) -- one warp each, lane l owns query
// columns [8l, 8l+8) of each half (dq/2 = 256):
//   dg_r  = w_r (dw_r - sum_r' w_r' dw_r')                    (softmax)
//   dS[p][h][t][i] = sum_{r: key_p(r) = i} dg_r              (dense, bf16)
//   dq^[t, h, :dq/2] = sum_i dS[0][h][t][i] K1[i],  dq^[t, h, dq/2:] = sum_j dS[1][h][t][j] K2[j]
//   (= sum_r dg_r K1[i_r] and sum_r dg_r K2[j_r]; dS in fp32 here)
// with i_r = id_r / K, j_r = id_r % K.  dS feeds the dK GEMMs; each warp
// writes its two dS rows whole -- zeros by coalesced 16-byte stores, then,
// after __syncwarp orders the lanes' stores, each nonzero (h, p, t, i) by one
// lane (duplicate keys of a row are combined with __match_any_sync first) --
// so no separate pass zeroes the 268 MB buffer (config 2).  K % 8 == 0.
template <int TOPK>
__global__ void __launch_bounds__(256) k_router_bwd(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                     const float* __restrict__ dw,
                                                     const __nv_bfloat16* __restrict__ keys,  // [2][K] rows
                                                     int64_t key_ld, __nv_bfloat16* __restrict__ dqhat,
                                                     __nv_bfloat16* __restrict__ dS, int T, int H, int K, int half) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int nl = half / 8;  // lanes covering one half in 8-column slices
  for (int th = gw; th < T * H; th += nw) {
    const int t = th / H, h = th - t * H;
    const int64_t o = static_cast<int64_t>(th) * TOPK;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint4* row = reinterpret_cast<uint4*>(dS + ((static_cast<int64_t>(p) * H + h) * T + t) * K);
      for (int c = lane; c < K / 8; c += 32) row[c] = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncwarp();
    // a selection whose id lies outside [0, K*K) (k_count_experts reports
    // it) contributes nothing and reads key row 0
    const int id_in = lane < TOPK ? ids[o + lane] : 0;
    const bool act = lane < TOPK && static_cast<unsigned>(id_in) < static_cast<unsigned>(K * K);
    const float wr = act ? w[o + lane] : 0.f;
    const float dwr = act ? dw[o + lane] : 0.f;
    float s = wr * dwr;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float dg = act ? wr * (dwr - s) : 0.f;
    const int id = act ? id_in : 0;
    const int i1 = id / K, i2 = id - i1 * K;
    // dS scatter: lanes with the same key combine (each lane walks the lanes
    // of its key group, the warp as long as the largest group), the lowest
    // lane of a group stores; the groups' keys, sums and leaders are kept for
    // dq^ below
    int key_p[2];
    float tot_p[2];
    unsigned lead_p[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int key = act ? (p == 0 ? i1 : i2) : -1 - lane;
      unsigned m = __match_any_sync(0xffffffffu, key);
      const int leader = __ffs(m) - 1;
      const int rounds = __reduce_max_sync(0xffffffffu, static_cast<unsigned>(__popc(m)));
      float tot = 0.f;
      for (int it = 0; it < rounds; ++it) {
        const int src = m ? __ffs(m) - 1 : lane;
        const float gu = __shfl_sync(0xffffffffu, dg, src);
        tot += m ? gu : 0.f;
        m &= m - 1u;
      }
      const bool lead = act && leader == lane;
      if (lead) dS[((static_cast<int64_t>(p) * H + h) * T + t) * K + key] = __float2bfloat16_rn(tot);
      key_p[p] = key;
      tot_p[p] = tot;
      lead_p[p] = __ballot_sync(0xffffffffu, lead);
    }
    // dq^_p = sum over the half's distinct sub-keys of dS * key row (the grid
    // top-k of a row draws on a few distinct sub-keys per half, ~5 of 16 at
    // k = 16); bf16 pairs widen to fp32 pairs by shifts
    unsigned long long acc[2][4];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[p][i] = 0ull;
      unsigned m = lead_p[p];
      while (m != 0u) {  // warp-uniform
        const int src = __ffs(m) - 1;
        m &= m - 1u;
        const float g = __shfl_sync(0xffffffffu, tot_p[p], src);
        const int kk = __shfl_sync(0xffffffffu, key_p[p], src);
        if (lane < nl) {
          const uint4 a =
              *reinterpret_cast<const uint4*>(keys + (static_cast<int64_t>(p) * K + kk) * key_ld + 8 * lane);
          const unsigned long long g2 = pk2(g, g);
          const uint32_t av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const unsigned long long fa = pk2(__uint_as_float(av[i] << 16), __uint_as_float(av[i] & 0xffff0000u));
            acc[p][i] = ffma2(g2, fa, acc[p][i]);
          }
        }
      }
    }
    if (lane < nl) {
      // dq^ is stored in bf16: it only feeds BatchNorm's backward, whose
      // output dq is the bf16 operand of the dx / dW_q GEMMs
      __nv_bfloat16* dst = dqhat + static_cast<int64_t>(t) * (H * 2 * half) + static_cast<int64_t>(h) * 2 * half;
      uint32_t o0[4], o1[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a0, a1, b0, b1;
        upk2(acc[0][i], a0, a1);
        upk2(acc[1][i], b0, b1);
        const __nv_bfloat162 pa = __floats2bfloat162_rn(a0, a1), pb = __floats2bfloat162_rn(b0, b1);
        o0[i] = *reinterpret_cast<const uint32_t*>(&pa);
        o1[i] = *reinterpret_cast<const uint32_t*>(&pb);
      }
      *reinterpret_cast<uint4*>(dst + 8 * lane) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
      *reinterpret_cast<uint4*>(dst + half + 8 * lane) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
    }
  }
}

// ------------------------------------------------------------------------
// BatchNorm backward.  x^ = (qpre - mean) * invstd (batch statistics in
// training mode, running statistics in eval mode).  Column sums over tokens
// of dq^ and dq^ * x^ (slab partials, then a finalize), then
//   train: dq = gamma*invstd*(dq^ - sum(dq^)/T - x^ * sum(dq^ x^)/T), dbias = 0
//   eval:  dq = gamma*invstd*dq^,                           dbias = sum(dq)
// dgamma = sum(dq^ x^), dbeta = sum(dq^).  dq is written as bf16 into the
// GEMM operand du[:, :C].  The apply pass evaluates
//   dq = A dq^ + B (qpre - mean) + D,  A = gamma*invstd, B = -A*invstd*m2,
//   D = -A*m1
// with coef[c] = (A, B, D, mean): centring qpre before the multiply keeps the
// cancellation exact where qpre and the mean agree to many bits.
__global__ void k_bn_bwd_partial(const float* __restrict__ dqh, const float* __restrict__ qpre,
                                 const float* __restrict__ mean, const float* __restrict__ invstd, int T, int C,
                                 float* __restrict__ part) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int slab = blockIdx.y;
  if (col >= C) return;
  const float mu = mean[col], is = invstd[col];
  const int r0 = slab * BN_ROWS_PER_SLAB;
  const int r1 = min(T, r0 + BN_ROWS_PER_SLAB);
  float s = 0.f, sx = 0.f;
#pragma unroll 8
  for (int r = r0; r < r1; ++r) {
    const int64_t o = static_cast<int64_t>(r) * C + col;
    const float g = dqh[o];
    s += g;
    sx = fmaf(g, (qpre[o] - mu) * is, sx);
  }
  part[(static_cast<int64_t>(slab) * C + col) * 2 + 0] = s;
  part[(static_cast<int64_t>(slab) * C + col) * 2 + 1] = sx;
}

// The same partial sums over a bf16 dq^ (the bf16 path), two adjacent
// columns per thread (C even) so a warp reads 128 contiguous bytes of dq^ and
// 256 of qpre per row.  Grid x covers the column pairs.
__global__ void k_bn_bwd_partial_bf16(const __nv_bfloat16* __restrict__ dqh, const float* __restrict__ qpre,
                                      const float* __restrict__ mean, const float* __restrict__ invstd, int T, int C,
                                      float* __restrict__ part) {
  const int col = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  const int slab = blockIdx.y;
  if (col >= C) return;
  const float mu0 = mean[col], mu1 = mean[col + 1], is0 = invstd[col], is1 = invstd[col + 1];
  const int r0 = slab * BN_ROWS_PER_SLAB;
  const int r1 = min(T, r0 + BN_ROWS_PER_SLAB);
  float s0 = 0.f, s1 = 0.f, sx0 = 0.f, sx1 = 0.f;
#pragma unroll 8
  for (int r = r0; r < r1; ++r) {
    const int64_t o = static_cast<int64_t>(r) * C + col;
    const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dqh + o));
    const float2 q = *reinterpret_cast<const float2*>(qpre + o);
    s0 += g.x;
    s1 += g.y;
    sx0 = fmaf(g.x, (q.x - mu0) * is0, sx0);
    sx1 = fmaf(g.y, (q.y - mu1) * is1, sx1);
  }
  *reinterpret_cast<float4*>(part + (static_cast<int64_t>(slab) * C + col) * 2) = make_float4(s0, sx0, s1, sx1);
}

__global__ void k_bn_bwd_finalize(const float* __restrict__ part, int slabs, int C, int T, int training,
                                  const float* __restrict__ gamma, const float* __restrict__ mean,
                                  const float* __restrict__ invstd,
                                  float* __restrict__ dgamma, float* __restrict__ dbeta, float* __restrict__ dbias,
                                  float* __restrict__ coef) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  double s = 0.0, sx = 0.0;
  for (int k = 0; k < slabs; ++k) {
    s += part[(static_cast<int64_t>(k) * C + col) * 2 + 0];
    sx += part[(static_cast<int64_t>(k) * C + col) * 2 + 1];
  }
  dgamma[col] = static_cast<float>(sx);
  dbeta[col] = static_cast<float>(s);
  const float gi = gamma[col] * invstd[col];
  // dq = gi * (dq^ - m1 - x^ * m2) with x^ = (qpre - mean) * invstd
  const float m1 = training ? static_cast<float>(s / T) : 0.f;
  const float m2 = training ? static_cast<float>(sx / T) : 0.f;
  dbias[col] = training ? 0.f : static_cast<float>(gi * s);
  const float B = -gi * m2 * invstd[col];
  reinterpret_cast<float4*>(coef)[col] = make_float4(gi, B, -gi * m1, mean[col]);
}

// One thread per 8 consecutive columns (C % 8 == 0), grid x over the column
// groups and y over the token rows (as k_bn_apply); coef[c] = (A, B, D, mean)
// from k_bn_bwd_finalize.
__global__ void k_bn_bwd_apply(const __nv_bfloat16* __restrict__ dqh, const float* __restrict__ qpre,
                               const float4* __restrict__ coef, int T, int C, __nv_bfloat16* __restrict__ du,
                               int64_t ldu) {
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= C) return;
  float4 k[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) k[u] = __ldg(coef + c0 + u);
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const int64_t o = static_cast<int64_t>(t) * C + c0;
    float gv[8];
    unpack_b8(*reinterpret_cast<const uint4*>(dqh + o), gv);
    const float4 q0 = *reinterpret_cast<const float4*>(qpre + o), q1 = *reinterpret_cast<const float4*>(qpre + o + 4);
    const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    uint32_t out[4];
#pragma unroll
    for (int u = 0; u < 8; u += 2) {
      const float r0 = fmaf(k[u].x, gv[u], fmaf(k[u].y, qv[u] - k[u].w, k[u].z));
      const float r1 = fmaf(k[u + 1].x, gv[u + 1], fmaf(k[u + 1].y, qv[u + 1] - k[u + 1].w, k[u + 1].z));
      const __nv_bfloat162 b = __floats2bfloat162_rn(r0, r1);
      out[u >> 1] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(du + static_cast<int64_t>(t) * ldu + c0) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

// Eval-mode statistics for the backward on qpre (which contains the bias):
// x^ = (qpre - running_mean) * 1/sqrt(running_var + eps).
__global__ void k_bn_eval_stats(const float* __restrict__ bn, int C, float eps, float* __restrict__ mean,
                                float* __restrict__ invstd) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  mean[col] = bn[3 * C + col];
  invstd[col] = 1.0f / sqrtf(bn[4 * C + col] + eps);
}

// out[c][j] = in[j][c] for an fp32 [rows, cols] matrix (small weight grads).
__global__ void k_transpose_f32(const float* __restrict__ in, int rows, int cols, float* __restrict__ out,
                                int64_t ldo) {
  __shared__ float tile[32][33];
  const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int r = by + j, c = bx + threadIdx.x;
    if (r < rows && c < cols) tile[j][threadIdx.x] = in[static_cast<int64_t>(r) * cols + c];
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int c = bx + j, r = by + threadIdx.x;
    if (c < cols && r < rows) out[static_cast<int64_t>(c) * ldo + r] = tile[threadIdx.x][j];
  }
}

}  // namespace ethos
