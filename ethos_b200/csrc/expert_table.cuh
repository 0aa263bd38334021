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
// Phase B is a gather: one warp per token streams the token's selected rows
// (coalesced 1 KB each) through a shared-memory cp.async ring; the dot
// products of each batch of rows are reduced across lanes with shuffles and
// the weighted sum stays in the lanes' registers.
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ethos {

constexpr int GATHER_WARPS = 8;
constexpr int GATHER_THREADS = GATHER_WARPS * 32;
constexpr int GATHER_ROWS = 4;     // table rows per batch
constexpr int GATHER_STAGES = 5;   // cp.async ring depth per warp (4 batches in flight)
constexpr int GATHER_STAGE_BYTES = GATHER_ROWS * 1024 + 16;          // rows + 4 routing weights
constexpr int GATHER_WARP_BYTES = GATHER_STAGES * GATHER_STAGE_BYTES + 2 * 2048;  // + 2 x_proj buffers
constexpr int GATHER_SMEM_BYTES = GATHER_WARPS * GATHER_WARP_BYTES;

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

// One warp walks tokens gw, gw + nw, ...; its rows are processed in batches of
// 4 through a 5-stage cp.async ring, so 4 batches (16 KB) per warp are in
// flight while one is reduced.  Lane l copies and later reads only its own
// slices of each row, hidden columns [8l, 8l + 8) and [256 + 8l, 256 + 8l + 8)
// (bytes [16l, 16l + 16) and [512 + 16l, ...)), so a cp.async.wait_group
// alone orders copy and use.  Needs R >= 16 (a token spans >= 4 batches, so
// the two x_proj buffers are never overwritten while in use).
__global__ void __launch_bounds__(GATHER_THREADS, 1)
    k_expert_gather(const __half* __restrict__ table, const int32_t* __restrict__ ids, const float* __restrict__ w,
                    const float* __restrict__ xp, __nv_bfloat16* __restrict__ hacc_out,
                    float* __restrict__ dot_out, int T, int R, int N, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  uint8_t* wbase = smem_raw + wib * GATHER_WARP_BYTES;
  uint8_t* xpbuf = wbase + GATHER_STAGES * GATHER_STAGE_BYTES;
  const int gw = blockIdx.x * GATHER_WARPS + wib;
  const int nw = gridDim.x * GATHER_WARPS;
  const int nbt = R / GATHER_ROWS;  // batches per token
  const int ntok = T > gw ? (T - 1 - gw) / nw + 1 : 0;
  const int nb = ntok * nbt;
  const int b3 = (lane >> 3) & 1, b4 = (lane >> 4) & 1;
  const int grp = (lane >> 3) & 3;  // row of the batch whose dot this lane ends up holding

  // ids of the next batch to issue, loaded one issue ahead (int4 broadcast)
  auto load_ids = [&](int b) -> int4 {
    if (b >= nb) return make_int4(0, 0, 0, 0);
    const int t = gw + (b / nbt) * nw;
    const int r0 = (b % nbt) * GATHER_ROWS;
    return __ldg(reinterpret_cast<const int4*>(ids + static_cast<int64_t>(t) * R + r0));
  };
  auto issue = [&](int b, int4 id4) {
    const int t = gw + (b / nbt) * nw;
    const int r0 = (b % nbt) * GATHER_ROWS;
    uint8_t* st = wbase + (b % GATHER_STAGES) * GATHER_STAGE_BYTES;
    const int idv[4] = {id4.x, id4.y, id4.z, id4.w};
#pragma unroll
    for (int u = 0; u < GATHER_ROWS; ++u) {
      int id = idv[u];
      if (id < 0 || id >= N) {
        if (lane == 0) record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
        id = 0;
      }
      const char* src = reinterpret_cast<const char*>(table + static_cast<int64_t>(id) * 512);
      cp_async_16(st + u * 1024 + 16 * lane, src + 16 * lane);
      cp_async_16(st + u * 1024 + 512 + 16 * lane, src + 512 + 16 * lane);
    }
    if (lane == 0) cp_async_16(st + GATHER_ROWS * 1024, w + static_cast<int64_t>(t) * R + r0);
    if (r0 == 0) {  // first batch of a token also brings this lane's x_proj slices
      const char* xs = reinterpret_cast<const char*>(xp + static_cast<int64_t>(t) * 512);
      uint8_t* xd = xpbuf + ((b / nbt) & 1) * 2048;
      cp_async_16(xd + 32 * lane, xs + 32 * lane);
      cp_async_16(xd + 32 * lane + 16, xs + 32 * lane + 16);
      cp_async_16(xd + 1024 + 32 * lane, xs + 1024 + 32 * lane);
      cp_async_16(xd + 1024 + 32 * lane + 16, xs + 1024 + 32 * lane + 16);
    }
  };

  int4 next_ids = load_ids(0);
#pragma unroll 1
  for (int b = 0; b < GATHER_STAGES - 1; ++b) {
    const int4 cur = next_ids;
    next_ids = load_ids(b + 1);
    if (b < nb) issue(b, cur);
    cp_async_commit();
  }
  float xv[16];
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll 1
  for (int b = 0; b < nb; ++b) {
    {
      const int bi = b + GATHER_STAGES - 1;
      const int4 cur = next_ids;
      next_ids = load_ids(bi + 1);
      if (bi < nb) issue(bi, cur);
      cp_async_commit();
    }
    cp_async_wait_group<GATHER_STAGES - 1>();
    const int t = gw + (b / nbt) * nw;
    const int r0 = (b % nbt) * GATHER_ROWS;
    const uint8_t* st = wbase + (b % GATHER_STAGES) * GATHER_STAGE_BYTES;
    if (r0 == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(xpbuf + ((b / nbt) & 1) * 2048);
      // this lane's x_proj columns [8l, 8l+8) and [256+8l, 256+8l+8)
      const float4 a0 = x4[2 * lane], a1 = x4[2 * lane + 1], c0 = x4[64 + 2 * lane], c1 = x4[64 + 2 * lane + 1];
      xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
      xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
      xv[8] = c0.x; xv[9] = c0.y; xv[10] = c0.z; xv[11] = c0.w;
      xv[12] = c1.x; xv[13] = c1.y; xv[14] = c1.z; xv[15] = c1.w;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    }
    uint4 hv[GATHER_ROWS][2];
    float part[GATHER_ROWS];
#pragma unroll
    for (int u = 0; u < GATHER_ROWS; ++u) {
      hv[u][0] = *reinterpret_cast<const uint4*>(st + u * 1024 + 16 * lane);
      hv[u][1] = *reinterpret_cast<const uint4*>(st + u * 1024 + 512 + 16 * lane);
      float f[8];
      float sacc = 0.f;
      unpack_h8(hv[u][0], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) sacc = fmaf(f[i], xv[i], sacc);
      unpack_h8(hv[u][1], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) sacc = fmaf(f[i], xv[8 + i], sacc);
      part[u] = sacc;
    }
    // transpose-reduce 4 partial dots over 32 lanes (6 shuffles): lanes
    // 8g..8g+7 end up with the full dot of row r0 + g
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
    float dot = part[0] + __shfl_xor_sync(0xffffffffu, part[0], 4);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    const float wgt = reinterpret_cast<const float*>(st + GATHER_ROWS * 1024)[grp];
    const float a_mine = gelu_erf(dot) * wgt;
    if (dot_out != nullptr && (lane & 7) == 0) dot_out[static_cast<int64_t>(t) * R + r0 + grp] = dot;
#pragma unroll
    for (int u = 0; u < GATHER_ROWS; ++u) {
      const float a = __shfl_sync(0xffffffffu, a_mine, 8 * u);
      float f[8];
      unpack_h8(hv[u][0], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(a, f[i], acc[i]);
      unpack_h8(hv[u][1], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[8 + i] = fmaf(a, f[i], acc[8 + i]);
    }
    if (r0 + GATHER_ROWS == R) {
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162 bb = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      __nv_bfloat16* dst = hacc_out + static_cast<int64_t>(t) * 512;
      *reinterpret_cast<uint4*>(dst + 8 * lane) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst + 256 + 8 * lane) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
  cp_async_wait_group<0>();
}

}  // namespace ethos
