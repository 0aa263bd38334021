// Expert-table execution of the reordered experts.
//
// h_i = gelu_erf(z_i @ W1^T) (model.py:323) depends only on the expert id, not
// on the token.  With T*H*k selections per step over N experts (2.1 M over
// 262 144 at the default size, ~8 per expert) it is cheaper to evaluate it
// once per expert:
//   phase A  H[e, :] = fp16(gelu_erf(E[e, :] @ W1^T))   tcgen05 GEMM with a
//            GELU epilogue (EpiGeluF16), N x 512 fp16 table
//   phase B  per token t: for each selection r, gather H[id_r] (1 KB rows),
//            dot_r = H[id_r] . xp_t, a_r = gelu_erf(dot_r) * w_r,
//            hacc_t = sum_r a_r H[id_r]                        (this kernel)
// Phase B is a gather: one warp per token, lane l owns hidden columns
// [16l, 16l + 16), so each selected row is one coalesced 1 KB load; the dot
// products of a batch of 8 rows are reduced across lanes with 9 shuffles and
// the weighted sum stays in the lanes' registers.
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ethos {

constexpr int GATHER_THREADS = 256;
constexpr int GATHER_BATCH = 8;

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void unpack_h8(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__global__ void __launch_bounds__(GATHER_THREADS, 1)
    k_expert_gather(const __half* __restrict__ table, const int32_t* __restrict__ ids, const float* __restrict__ w,
                    const float* __restrict__ xp, __nv_bfloat16* __restrict__ hacc_out,
                    float* __restrict__ dot_out, int T, int R, int N, int* err) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
  const int grp = lane >> 2;  // row of the batch whose dot this lane ends up holding
  for (int t = gw; t < T; t += nw) {
    float xv[16];
    const float4* xs = reinterpret_cast<const float4*>(xp + static_cast<int64_t>(t) * 512 + lane * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = __ldg(xs + i);
      xv[4 * i] = f.x;
      xv[4 * i + 1] = f.y;
      xv[4 * i + 2] = f.z;
      xv[4 * i + 3] = f.w;
    }
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    const int32_t* idr = ids + static_cast<int64_t>(t) * R;
    const float* wr = w + static_cast<int64_t>(t) * R;
    for (int r0 = 0; r0 < R; r0 += GATHER_BATCH) {
      uint4 hv[GATHER_BATCH][2];
#pragma unroll
      for (int u = 0; u < GATHER_BATCH; ++u) {
        const int r = r0 + u;
        int id = r < R ? __ldg(idr + r) : 0;
        if (id < 0 || id >= N) {
          if (lane == 0) record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
          id = 0;
        }
        const char* src = reinterpret_cast<const char*>(table + static_cast<int64_t>(id) * 512 + lane * 16);
        hv[u][0] = ldg_nc_v4(src);
        hv[u][1] = ldg_nc_v4(src + 16);
      }
      float part[GATHER_BATCH];
#pragma unroll
      for (int u = 0; u < GATHER_BATCH; ++u) {
        float f[8];
        float s = 0.f;
        unpack_h8(hv[u][0], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) s = fmaf(f[i], xv[i], s);
        unpack_h8(hv[u][1], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) s = fmaf(f[i], xv[8 + i], s);
        part[u] = s;
      }
      // transpose-reduce 8 partial dots over 32 lanes (9 shuffles): lanes
      // 4g..4g+3 end up with the full dot of row r0 + g
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = b4 ? part[i] : part[i + 4];
        const float keep = b4 ? part[i + 4] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = b3 ? part[i] : part[i + 2];
        const float keep = b3 ? part[i + 2] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      {
        const float send = b2 ? part[0] : part[1];
        const float keep = b2 ? part[1] : part[0];
        part[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      float dot = part[0] + __shfl_xor_sync(0xffffffffu, part[0], 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      const int rg = r0 + grp;
      const float a_mine = rg < R ? gelu_erf(dot) * __ldg(wr + rg) : 0.f;
      if (dot_out != nullptr && (lane & 3) == 0 && rg < R) dot_out[static_cast<int64_t>(t) * R + rg] = dot;
#pragma unroll
      for (int u = 0; u < GATHER_BATCH; ++u) {
        const float a = __shfl_sync(0xffffffffu, a_mine, 4 * u);
        float f[8];
        unpack_h8(hv[u][0], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(a, f[i], acc[i]);
        unpack_h8(hv[u][1], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[8 + i] = fmaf(a, f[i], acc[8 + i]);
      }
    }
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
    uint4* dst = reinterpret_cast<uint4*>(hacc_out + static_cast<int64_t>(t) * 512 + lane * 16);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

}  // namespace ethos
