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

// 16 warps x 2 stages: the kernel is bound by load latency per warp, so
// resident warps matter more than ring depth (measured on B200 at 16384
// tokens x 128 selections: 8x5 0.47 ms, 12x3 0.40, 14x3 0.36, 16x2 0.31;
// 18 and more warps spill registers).  Restricting the routed ids to an
// L2-resident eighth of the table saves only 6 %: the per-SM copy and
// arithmetic pipeline binds, not DRAM.
#ifndef ETHOS_GATHER_WARPS
#define ETHOS_GATHER_WARPS 16
#endif
#ifndef ETHOS_GATHER_STAGES
#define ETHOS_GATHER_STAGES 2
#endif
constexpr int GATHER_WARPS = ETHOS_GATHER_WARPS;
constexpr int GATHER_THREADS = GATHER_WARPS * 32;
constexpr int GATHER_ROWS = 4;                     // table rows per batch
constexpr int GATHER_STAGES = ETHOS_GATHER_STAGES; // cp.async ring depth per warp
constexpr int GATHER_STAGE_BYTES = GATHER_ROWS * 1024 + 16;          // rows + 4 routing weights
// + one x_proj buffer: a token's x_proj moves to registers at its first batch,
// and the next token's copy is issued at least one batch later (R/4 > STAGES-1)
// (the table path runs with R >= 16 selections per token, i.e. 4 batches)
// ETHOS_GATHER_XP_REGS (the default): a token's x_proj row is loaded straight
// into the lanes' registers at its first batch instead of through a
// shared-memory buffer (0.266 against 0.270 ms at 16 384 tokens; the 2 KB per
// warp it frees did not pay as a third ring stage: 16 x 3 0.269 ms, 14 x 4
// 0.286 ms, 15 x 3 with the buffer 0.285 ms).
#ifndef ETHOS_GATHER_XP_REGS
#define ETHOS_GATHER_XP_REGS 1
#endif
constexpr int GATHER_XP_BYTES = ETHOS_GATHER_XP_REGS ? 0 : 2048;
constexpr int GATHER_WARP_BYTES = GATHER_STAGES * GATHER_STAGE_BYTES + GATHER_XP_BYTES;
constexpr int GATHER_SMEM_BYTES = GATHER_WARPS * GATHER_WARP_BYTES;
static_assert(GATHER_STAGES >= 2 && (ETHOS_GATHER_XP_REGS || GATHER_STAGES <= 4),
              "single x_proj buffer needs STAGES-1 < 4 batches");
static_assert(GATHER_SMEM_BYTES <= 227 * 1024, "gather ring exceeds shared memory");

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 8 fp16 (one uint4) -> 4 packed fp32 pairs
__device__ __forceinline__ void unpack_h8_x2(const uint4& u, unsigned long long* p) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(h[i]);
    p[i] = pk2(v.x, v.y);
  }
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
// 4 through a GATHER_STAGES-deep cp.async ring (2 stages by default), so
// GATHER_STAGES - 1 batches (4 KB each) per warp are in flight while one is
// reduced; the token's x_proj slices move to registers at its first batch.
// Lane l copies and later reads only its own slices of each row, hidden
// columns [8l, 8l + 8) and [256 + 8l, 256 + 8l + 8) (bytes [16l, 16l + 16)
// and [512 + 16l, ...)), so a cp.async.wait_group alone orders copy and use.
// With the shared x_proj buffer (ETHOS_GATHER_XP_REGS 0) it needs
// R / 4 > STAGES - 1, so that a token's x_proj is read into registers before
// the next token's copy is issued.
__global__ void __launch_bounds__(GATHER_THREADS, 1)
    k_expert_gather(const __half* __restrict__ table, const int32_t* __restrict__ ids, const float* __restrict__ w,
                    const float* __restrict__ xp, __nv_bfloat16* __restrict__ hacc_out,
                    float* __restrict__ dot_out, int T, int R, int N, int* err) {
  pdl_launch_dependents();
  pdl_wait();
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

  // Cursors instead of div/mod by the runtime batch count: the issue cursor
  // (token it_t, row it_r) runs STAGES-1 batches ahead of the consume cursor.
  int it_t = gw, it_r = 0, it_n = 0;
  bool bad_id = false;
  // ids of the batch at the issue cursor, loaded one issue ahead (int4 broadcast)
  int4 next_ids = nb > 0 ? __ldg(reinterpret_cast<const int4*>(ids + static_cast<int64_t>(gw) * R))
                         : make_int4(0, 0, 0, 0);
  auto issue_next = [&]() {
    if (it_n < nb) {
      const int t = it_t, r0 = it_r;
      uint8_t* st = wbase + (static_cast<unsigned>(it_n) % GATHER_STAGES) * GATHER_STAGE_BYTES;
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
      if (!ETHOS_GATHER_XP_REGS && r0 == 0) {  // first batch of a token also brings this lane's x_proj slices
        const char* xs = reinterpret_cast<const char*>(xp + static_cast<int64_t>(t) * 512);
        cp_async_16(xpbuf + 32 * lane, xs + 32 * lane);
        cp_async_16(xpbuf + 32 * lane + 16, xs + 32 * lane + 16);
        cp_async_16(xpbuf + 1024 + 32 * lane, xs + 1024 + 32 * lane);
        cp_async_16(xpbuf + 1024 + 32 * lane + 16, xs + 1024 + 32 * lane + 16);
      }
      // advance the issue cursor and prefetch its ids
      ++it_n;
      it_r += GATHER_ROWS;
      if (it_r == R) {
        it_r = 0;
        it_t += nw;
      }
      if (it_n < nb) next_ids = __ldg(reinterpret_cast<const int4*>(ids + static_cast<int64_t>(it_t) * R + it_r));
    }
    cp_async_commit();
  };

#pragma unroll 1
  for (int b = 0; b < GATHER_STAGES - 1; ++b) issue_next();
  unsigned long long xv2[8];   // this lane's x_proj columns as packed pairs
  unsigned long long acc2[8];  // hacc columns as packed pairs
#pragma unroll
  for (int i = 0; i < 8; ++i) acc2[i] = 0ull;
  int t = gw, r0 = 0;  // consume cursor
#pragma unroll 1
  for (int b = 0; b < nb; ++b) {
    issue_next();
    cp_async_wait_group<GATHER_STAGES - 1>();
    const uint8_t* st = wbase + (static_cast<unsigned>(b) % GATHER_STAGES) * GATHER_STAGE_BYTES;
    if (r0 == 0) {
      const float4* x4 = ETHOS_GATHER_XP_REGS ? reinterpret_cast<const float4*>(xp + static_cast<int64_t>(t) * 512)
                                              : reinterpret_cast<const float4*>(xpbuf);
      // this lane's x_proj columns [8l, 8l+8) and [256+8l, 256+8l+8)
      const float4 a0 = x4[2 * lane], a1 = x4[2 * lane + 1], c0 = x4[64 + 2 * lane], c1 = x4[64 + 2 * lane + 1];
      xv2[0] = pk2(a0.x, a0.y); xv2[1] = pk2(a0.z, a0.w); xv2[2] = pk2(a1.x, a1.y); xv2[3] = pk2(a1.z, a1.w);
      xv2[4] = pk2(c0.x, c0.y); xv2[5] = pk2(c0.z, c0.w); xv2[6] = pk2(c1.x, c1.y); xv2[7] = pk2(c1.z, c1.w);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc2[i] = 0ull;
    }
    // rows are unpacked to fp32 pairs once and kept for the weighted sum
    unsigned long long hf[GATHER_ROWS][8];
    float part[GATHER_ROWS];
#pragma unroll
    for (int u = 0; u < GATHER_ROWS; ++u) {
      unpack_h8_x2(*reinterpret_cast<const uint4*>(st + u * 1024 + 16 * lane), hf[u]);
      unpack_h8_x2(*reinterpret_cast<const uint4*>(st + u * 1024 + 512 + 16 * lane), hf[u] + 4);
      unsigned long long s2 = 0ull;
#pragma unroll
      for (int i = 0; i < 8; ++i) s2 = ffma2(hf[u][i], xv2[i], s2);
      float lo, hi;
      upk2(s2, lo, hi);
      part[u] = lo + hi;
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
      const unsigned long long a2 = pk2(a, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc2[i] = ffma2(a2, hf[u][i], acc2[i]);
    }
    if (r0 + GATHER_ROWS == R) {
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float lo, hi;
        upk2(acc2[i], lo, hi);
        const __nv_bfloat162 bb = __floats2bfloat162_rn(lo, hi);
        o[i] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      __nv_bfloat16* dst = hacc_out + static_cast<int64_t>(t) * 512;
      *reinterpret_cast<uint4*>(dst + 8 * lane) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst + 256 + 8 * lane) = make_uint4(o[4], o[5], o[6], o[7]);
    }
    r0 += GATHER_ROWS;
    if (r0 == R) {
      r0 = 0;
      t += nw;
    }
  }
  cp_async_wait_group<0>();
  if (__any_sync(0xffffffffu, bad_id) && lane == 0) record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
}

}  // namespace ethos
