// Persistent tcgen05 GEMM  D[M, N] = A[M, K] * B[N, K]^T  (bf16 in, fp32 TMEM
// accumulate) with a pluggable per-row epilogue.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..9 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31;
// warps 2-5 take columns 0-127 of the tile, warps 6-9 columns 128-255).
// Tiles are 128 x 256 x 64 with a 4-stage TMA ring (48 KB per stage, 128-byte
// swizzle) and two 256-column TMEM accumulators, so the epilogue of tile i
// overlaps the main loop of tile i+1.
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ethos {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 256;
constexpr int GEMM_BK = 64;
constexpr int GEMM_STAGES = 4;
constexpr int GEMM_A_BYTES = GEMM_BM * GEMM_BK * 2;
constexpr int GEMM_B_BYTES = GEMM_BN * GEMM_BK * 2;
constexpr int GEMM_STAGE_BYTES = GEMM_A_BYTES + GEMM_B_BYTES;
constexpr int GEMM_THREADS = 320;
constexpr int GEMM_EPI_THREADS = 256;

struct GemmCtl {
  uint64_t full[GEMM_STAGES];
  uint64_t empty[GEMM_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr int GEMM_SMEM_BYTES = GEMM_STAGES * GEMM_STAGE_BYTES + 1024 + static_cast<int>(sizeof(GemmCtl));

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// ------------------------------------------------------------- epilogues --
// Each functor is called per warp-chunk: `row` is this lane's output row and
// v[0..31] the fp32 accumulators of columns col..col+31.  Rows >= M must be
// ignored by the functor.

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// out[row, col] = bf16(scale * v)   (row-major, leading dimension ldo)
struct EpiStoreBF16 {
  __nv_bfloat16* out;
  int64_t ldo;
  int M;
  float scale;
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32]) const {
    if (row >= M) return;
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * ldo + col);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 u;
      u.x = pack_bf16x2(v[8 * j + 0] * scale, v[8 * j + 1] * scale);
      u.y = pack_bf16x2(v[8 * j + 2] * scale, v[8 * j + 3] * scale);
      u.z = pack_bf16x2(v[8 * j + 4] * scale, v[8 * j + 5] * scale);
      u.w = pack_bf16x2(v[8 * j + 6] * scale, v[8 * j + 7] * scale);
      dst[j] = u;
    }
  }
};

// out[row, col] = scale * v  (fp32), or += when accumulate != 0
struct EpiStoreF32 {
  float* out;
  int64_t ldo;
  int M;
  float scale;
  int accumulate;
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32]) const {
    if (row >= M) return;
    float4* dst = reinterpret_cast<float4*>(out + static_cast<int64_t>(row) * ldo + col);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 o = make_float4(v[4 * j] * scale, v[4 * j + 1] * scale, v[4 * j + 2] * scale, v[4 * j + 3] * scale);
      if (accumulate) {
        const float4 p = dst[j];
        o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
      }
      dst[j] = o;
    }
  }
};

// Router query projection + token projection sharing one A operand (x):
// columns [0, HQ) are the H heads' queries (query_projs, model.py:215),
// columns [HQ, HQ + dh) are x_proj = x @ W_u (model.py:326).
//  mode 0 (BatchNorm eval): q_hat = v * scale + offset, with the bias and the
//    running statistics folded into (scale, offset) per column, is written as
//    a bf16 hi/lo pair into the scoring operand
//    qs[(h*2 + half)][row][0..dq/2) = hi, [dq/2..dq) = lo.
//  mode 1 (BatchNorm train): qpre[row][col] = v + bias (fp32) for the batch
//    statistics pass.
// x_proj is always written fp32 to xp[row][0..dh).
struct EpiProj {
  int M;   // tokens
  int HQ;  // H * d_query
  int dq;
  int dh;
  int mode;
  const float* bias;    // [HQ]
  const float2* colp;   // [HQ] (scale, offset) for mode 0
  __nv_bfloat16* qs;
  float* qpre;
  float* xp;
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32]) const {
    if (row >= M) return;
    if (col >= HQ) {
      float4* dst = reinterpret_cast<float4*>(xp + static_cast<int64_t>(row) * dh + (col - HQ));
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      return;
    }
    if (mode == 1) {
      float4* dst = reinterpret_cast<float4*>(qpre + static_cast<int64_t>(row) * HQ + col);
      const float4* b4 = reinterpret_cast<const float4*>(bias + col);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 b = __ldg(b4 + j);
        dst[j] = make_float4(v[4 * j] + b.x, v[4 * j + 1] + b.y, v[4 * j + 2] + b.z, v[4 * j + 3] + b.w);
      }
      return;
    }
    const int h = col / dq;
    const int e = col - h * dq;
    const int half = dq >> 1;
    const int p = e >= half ? 1 : 0;
    const int i0 = e - p * half;
    __nv_bfloat16* base = qs + (static_cast<int64_t>(h * 2 + p) * M + row) * dq;
    const float4* cp4 = reinterpret_cast<const float4*>(colp + col);
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 c = __ldg(cp4 + i);
      const float q0 = fmaf(v[2 * i], c.x, c.y);
      const float q1 = fmaf(v[2 * i + 1], c.z, c.w);
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(q0, q1);
      const float2 hf = __bfloat1622float2(h2);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(q0 - hf.x, q1 - hf.y);
      hi[i] = *reinterpret_cast<const uint32_t*>(&h2);
      lo[i] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    uint4* dh_ = reinterpret_cast<uint4*>(base + i0);
    uint4* dl_ = reinterpret_cast<uint4*>(base + half + i0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dh_[j] = make_uint4(hi[4 * j], hi[4 * j + 1], hi[4 * j + 2], hi[4 * j + 3]);
      dl_[j] = make_uint4(lo[4 * j], lo[4 * j + 1], lo[4 * j + 2], lo[4 * j + 3]);
    }
  }
};

// Expert hidden table: out[row][col] = fp16(gelu_erf(v)) for the expert-
// expansion GEMM E @ W1^T (row = expert id, col = hidden unit; model.py:323
// evaluated once per expert instead of once per selection).
struct EpiGeluF16 {
  __half* out;
  int64_t ldo;
  int M;
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32]) const {
    if (row >= M) return;
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * ldo + col);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __half2 hh = __floats2half2_rn(gelu_erf(v[8 * j + 2 * u]), gelu_erf(v[8 * j + 2 * u + 1]));
        w[u] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
};

// ---------------------------------------------------------------- kernel --
template <class Epi>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_bf16_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, Epi epi, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  GemmCtl* ctl = reinterpret_cast<GemmCtl*>(smem + GEMM_STAGES * GEMM_STAGE_BYTES);
  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = N / GEMM_BN;
  const int num_tiles = num_m * num_n;
  const int num_k = K / GEMM_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GEMM_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], GEMM_EPI_THREADS);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      RingPos rp;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / num_n) * GEMM_BM;
        const int n0 = (tile % num_n) * GEMM_BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&ctl->empty[rp.stage], rp.phase ^ 1u, abort, err, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + rp.stage * GEMM_STAGE_BYTES;
          mbar_arrive_expect_tx(&ctl->full[rp.stage], GEMM_STAGE_BYTES);
          tma_load_2d(sa, &tmA, &ctl->full[rp.stage], kb * GEMM_BK, m0);
          tma_load_2d(sa + GEMM_A_BYTES, &tmB, &ctl->full[rp.stage], kb * GEMM_BK, n0);
          rp.advance(GEMM_STAGES);
        }
      }
      if (!ok) rp.drain(ctl->full, GEMM_STAGES, err, 5);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(GEMM_BM, GEMM_BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;  // false once this role gave up (abort or timeout)
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
        if (!mbar_wait(&ctl->acc_empty[buf], acc_phase ^ 1u, abort, err, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * GEMM_BN);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort, err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * GEMM_STAGE_BYTES);
          const uint32_t b_base = a_base + GEMM_A_BYTES;
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            umma_bf16(d, umma_desc_sw128(a_base + k * 32), umma_desc_sw128(b_base + k * 32), idesc,
                      (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&ctl->empty[stage]);
          if (++stage == GEMM_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&ctl->acc_full[buf]);
      }
      if (!ok || *abort) {
        // Drain: wait until every MMA this thread issued has completed.
        umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr, err, 6);
      }
    }
  } else {
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;  // column half of the tile
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
      const int m0 = (tile / num_n) * GEMM_BM;
      const int n0 = (tile % num_n) * GEMM_BN;
      const bool ok = mbar_wait(&ctl->acc_full[buf], acc_phase, abort, err, 4);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = ch * 4; c < ch * 4 + 4; ++c) {
        float v[32];
        tmem_ld32(tmem_addr(tmem, q * 32, buf * GEMM_BN + c * 32), v);
        epi(row, n0 + c * 32, v);
      }
      tc_fence_before();
      mbar_arrive(&ctl->acc_empty[buf]);
    }
  }

  // Teardown: on the normal path the epilogue consumed every committed
  // accumulator; on the abort path the producer and the MMA issuer drained
  // their in-flight copies and MMAs above.
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace ethos
