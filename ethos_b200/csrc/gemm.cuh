// Persistent tcgen05 GEMM  D[M, N] = sum_k A[m, k] * B[n, k]  (bf16 in, fp32
// TMEM accumulate) with a pluggable per-row epilogue.
//
// Operands are either K-major (stored [M][K] / [N][K], K contiguous) or
// MN-major (stored [K][M] / [K][N], M/N contiguous -- a transposed operand
// read in place).  Both are staged by TMA with the 128-byte swizzle:
//   K-major:  one box of 64 K x rows; UMMA steps K by 32 B inside the atom.
//   MN-major: boxes of 64 M/N x 64 K (8 KB, MN blocks 8 KB apart = LBO),
//             8-row K groups 1024 B apart (SBO); UMMA steps K by 2 KB.
// `hold_unit` >= 0 withholds one work unit's operand loads (a test of the
// bounded waits, see ethos_test_gemm_withhold); production launches pass -1.
// Roles: warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer, warps
// 2.. = 8 or 16 epilogue warps (warp w reads TMEM lanes 32*(w%4)..+31; each
// run of four consecutive warps takes one column group of the tile).
// Tiles are 128 x BN x 64 (BN = 128 or 256) with a TMA ring and two BN-column
// TMEM accumulators, so the epilogue of tile i overlaps the main loop of tile
// i+1.  Split-K: work unit u covers tile u % tiles and K blocks of slice
// u / tiles; split-K epilogues reduce into fp32 with vector atomics.
// Epilogues store through the LSU (per-row or warp-transposed rows), or, with
// Epi::kTmaStore (the expert-table GELU epilogues), stage each warp's 32-row
// block in shared memory and write it with TMA stores (tensor maps tmC, tmD).
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ethos {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 256;  // widest N tile
constexpr int GEMM_BK = 64;
constexpr int GEMM_STAGES = 4;
constexpr int GEMM_A_BYTES = GEMM_BM * GEMM_BK * 2;
constexpr int GEMM_B_BYTES = GEMM_BN * GEMM_BK * 2;
constexpr int GEMM_STAGE_BYTES = GEMM_A_BYTES + GEMM_B_BYTES;

struct GemmCtl {
  uint64_t full[GEMM_STAGES];
  uint64_t empty[GEMM_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr int GEMM_COLP_BYTES = 2 * 256 * 8;  // double-buffered per-tile column side data
constexpr int GEMM_STG_WARP_BYTES = 32 * 64;   // per epilogue warp: 32 rows x 64 B store staging

// Launch shape of the kernel for an epilogue: Epi::kEpiWarps epilogue warps
// (8, or 16 for arithmetic-heavy epilogues, which then overlap their
// arithmetic, TMEM reads and stores across more warps), and the TMA ring
// depth that fits next to their staging buffers.
template <class Epi>
struct GemmCfg {
  static constexpr int kEpiWarps = Epi::kEpiWarps;
  static_assert(kEpiWarps == 8 || kEpiWarps == 16, "8 or 16 epilogue warps");
  static constexpr int kEpiThreads = 32 * kEpiWarps;
  static constexpr int kThreads = 64 + kEpiThreads;
  // a TMA-store epilogue stages its warp's whole 32-row x 128-byte block of
  // each output (one or two outputs, tensor maps tmC and tmD); with two, the
  // ring keeps two stages (one tile's K = 128 here) to make room for them
  static constexpr int kTmaOutputs = Epi::kTmaStore ? Epi::kTmaOutputs : 0;
  static constexpr int kStages = kEpiWarps == 16 ? (kTmaOutputs == 2 ? 2 : 3) : GEMM_STAGES;
  static constexpr int kStgWarpBytes = Epi::kTmaStore ? 32 * 128 * kTmaOutputs : GEMM_STG_WARP_BYTES;
  static constexpr int kColpBytes = Epi::kColParamBytes > 0 ? GEMM_COLP_BYTES : 0;
  static constexpr int kSmem = kStages * GEMM_STAGE_BYTES + kColpBytes + kEpiWarps * kStgWarpBytes + 1024 +
                               static_cast<int>(sizeof(GemmCtl));
  static_assert(kSmem <= 227 * 1024, "GEMM shared memory");
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// ------------------------------------------------------------- epilogues --
// Per-warp context of an epilogue call: the warp's 32 output rows start at
// row0 (nrows of them are inside the matrix) and `stg` is its staging buffer
// (2 KB, or the 4 KB block of each output of a TMA-store epilogue).  All 32
// lanes call the functor together.
struct EpiCtx {
  uint8_t* stg;
  int row0;
  int nrows;
  int lane;
  int chunk;  // index of the 32-column chunk among this warp's chunks of the tile
};

// Warp-cooperative store of 32 rows x 64 bytes.  Lane l holds the 64 bytes
// of row row0 + l in w[0..3]; they pass through the staging buffer (16-byte
// pieces XOR-swizzled by (row >> 1) & 3, so both phases are free of bank
// conflicts) and each store instruction then writes 8 rows x 64 contiguous
// bytes instead of 32 scattered 16-byte pieces.
__device__ __forceinline__ void warp_store_rows64(const EpiCtx& cx, const uint4 (&w)[4], char* dst_row0,
                                                  int64_t stride) {
  const int l = cx.lane;
  const int sw = (l >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(cx.stg + l * 64 + ((j ^ sw) << 4)) = w[j];
  __syncwarp();
  const int piece = l & 3;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (l >> 2);
    const uint4 u = *reinterpret_cast<const uint4*>(cx.stg + r * 64 + ((piece ^ ((r >> 1) & 3)) << 4));
    if (r < cx.nrows) *reinterpret_cast<uint4*>(dst_row0 + r * stride + piece * 16) = u;
  }
  __syncwarp();
}

// Each functor is called per warp-chunk: `row` is this lane's output row and
// v[0..31] the fp32 accumulators of columns col..col+31.  Rows >= M must be
// ignored by the functor.  A functor with per-column side data declares
// kColParamBytes > 0 and load_col_params(): before each tile's accumulator is
// read, the epilogue warps stage the tile's 256 columns of side data into
// shared memory (double-buffered) and operator() receives it as `cp`
// (indexed by column - n0).
struct EpiNoColParams {
  static constexpr int kColParamBytes = 0;
  static constexpr int kEpiWarps = 8;
  // true: the functor writes its fp16/bf16 row pieces into the warp's staging
  // block (EpiCtx::stg, 32 rows x 128 B, 128-byte swizzle) and the kernel
  // stores the block with one TMA store per warp and tile (tensor map tmC)
  static constexpr bool kTmaStore = false;
  static constexpr int kTmaOutputs = 1;
  __device__ __forceinline__ void load_col_params(int, uint8_t*, int) const {}
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// out[row, col] = bf16(scale * v)   (row-major, leading dimension ldo)
struct EpiStoreBF16 : EpiNoColParams {
  __nv_bfloat16* out;
  int64_t ldo;
  int M;
  float scale;
  __device__ __forceinline__ void operator()(int, int col, float (&v)[32], const uint8_t*, const EpiCtx& cx) const {
    uint4 w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      w[j].x = pack_bf16x2(v[8 * j + 0] * scale, v[8 * j + 1] * scale);
      w[j].y = pack_bf16x2(v[8 * j + 2] * scale, v[8 * j + 3] * scale);
      w[j].z = pack_bf16x2(v[8 * j + 4] * scale, v[8 * j + 5] * scale);
      w[j].w = pack_bf16x2(v[8 * j + 6] * scale, v[8 * j + 7] * scale);
    }
    warp_store_rows64(cx, w, reinterpret_cast<char*>(out + static_cast<int64_t>(cx.row0) * ldo + col), ldo * 2);
  }
};

// out[row, col] = scale * v  (fp32), or += when accumulate != 0
struct EpiStoreF32 : EpiNoColParams {
  float* out;
  int64_t ldo;
  int M;
  float scale;
  int accumulate;
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32], const uint8_t*, const EpiCtx&) const {
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

// out[row, col] += scale * v  with fp32 vector atomics (split-K partials,
// gradient accumulation)
struct EpiAtomicF32 : EpiNoColParams {
  float* out;
  int64_t ldo;
  int M;
  float scale;
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32], const uint8_t*, const EpiCtx&) const {
    if (row >= M) return;
    float* dst = out + static_cast<int64_t>(row) * ldo + col;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(dst + 4 * j), "f"(v[4 * j] * scale),
                   "f"(v[4 * j + 1] * scale), "f"(v[4 * j + 2] * scale), "f"(v[4 * j + 3] * scale)
                   : "memory");
    }
  }
};

// Router query projection + token projection sharing one A operand (x):
// columns [0, HQ) are the H heads' queries (query_projs, model.py:215),
// columns [HQ, HQ + dh) are x_proj = x @ W_u (model.py:326).
//  mode 0 (BatchNorm eval): q_hat = v * scale + offset, with the bias and the
//    running statistics folded into (scale, offset) per column, is written as
//    a bf16 hi/lo pair into the scoring operand
//    qs[half][h][row][0..dq/2) = hi, [dq/2..dq) = lo.
//  mode 1 (BatchNorm train): qpre[row][col] = v + bias (fp32) for the batch
//    statistics pass.
// x_proj is always written fp32 to xp[row][0..dh).  With `part` set, the fp32
// partial sum part[row][col] of an earlier launch over other K columns is
// added to v first (a contraction split over launches, each accumulating from
// zero in TMEM).
struct EpiProj {
  static constexpr int kColParamBytes = 8;  // float2 (scale, offset) or (bias, -)
  static constexpr int kEpiWarps = 8;
  static constexpr bool kTmaStore = false;
  static constexpr int kTmaOutputs = 1;
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
  const float* part;  // [M][ldp] or nullptr
  int64_t ldp;
  // epilogue thread `tid` (0..255) stages column n0 + tid
  __device__ __forceinline__ void load_col_params(int n0, uint8_t* dst, int tid) const {
    const int col = n0 + tid;
    float2 v = make_float2(0.f, 0.f);
    if (col < HQ) v = mode == 1 ? make_float2(__ldg(bias + col), 0.f) : __ldg(colp + col);
    reinterpret_cast<float2*>(dst)[tid] = v;
  }
  __device__ __forceinline__ void operator()(int row, int col, float (&v)[32], const uint8_t* cp,
                                             const EpiCtx& cx) const {
    if (part != nullptr && row < M) {
      const float4* src = reinterpret_cast<const float4*>(part + static_cast<int64_t>(row) * ldp + col);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 a = __ldg(src + j);
        v[4 * j] += a.x;
        v[4 * j + 1] += a.y;
        v[4 * j + 2] += a.z;
        v[4 * j + 3] += a.w;
      }
    }
    if (col >= HQ) {
      char* dst = reinterpret_cast<char*>(xp + static_cast<int64_t>(cx.row0) * dh + (col - HQ));
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        uint4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w[j] = make_uint4(__float_as_uint(v[16 * hlf + 4 * j]), __float_as_uint(v[16 * hlf + 4 * j + 1]),
                            __float_as_uint(v[16 * hlf + 4 * j + 2]), __float_as_uint(v[16 * hlf + 4 * j + 3]));
        warp_store_rows64(cx, w, dst + 64 * hlf, static_cast<int64_t>(dh) * 4);
      }
      return;
    }
    const float2* cpc = reinterpret_cast<const float2*>(cp) + (col & 255);
    if (mode == 1) {
      char* dst = reinterpret_cast<char*>(qpre + static_cast<int64_t>(cx.row0) * HQ + col);
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        uint4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int b = 16 * hlf + 4 * j;
          w[j] = make_uint4(__float_as_uint(v[b] + cpc[b].x), __float_as_uint(v[b + 1] + cpc[b + 1].x),
                            __float_as_uint(v[b + 2] + cpc[b + 2].x), __float_as_uint(v[b + 3] + cpc[b + 3].x));
        }
        warp_store_rows64(cx, w, dst + 64 * hlf, static_cast<int64_t>(HQ) * 4);
      }
      return;
    }
    const int h = col / dq;
    const int e = col - h * dq;
    const int half = dq >> 1;
    const int p = e >= half ? 1 : 0;
    const int i0 = e - p * half;
    __nv_bfloat16* base = qs + (static_cast<int64_t>(p * (HQ / dq) + h) * M + cx.row0) * dq;
    const float4* cp4 = reinterpret_cast<const float4*>(cpc);
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 c = cp4[i];
      const float q0 = fmaf(v[2 * i], c.x, c.y);
      const float q1 = fmaf(v[2 * i + 1], c.z, c.w);
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(q0, q1);
      const float2 hf = __bfloat1622float2(h2);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(q0 - hf.x, q1 - hf.y);
      hi[i] = *reinterpret_cast<const uint32_t*>(&h2);
      lo[i] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    uint4 wh[4], wl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wh[j] = make_uint4(hi[4 * j], hi[4 * j + 1], hi[4 * j + 2], hi[4 * j + 3]);
      wl[j] = make_uint4(lo[4 * j], lo[4 * j + 1], lo[4 * j + 2], lo[4 * j + 3]);
    }
    warp_store_rows64(cx, wh, reinterpret_cast<char*>(base + i0), static_cast<int64_t>(dq) * 2);
    warp_store_rows64(cx, wl, reinterpret_cast<char*>(base + half + i0), static_cast<int64_t>(dq) * 2);
  }
};

// Lane r's 64 bytes w[0..3] of chunk `chunk` into its row of a staged 32 x 64
// fp16 block: 16-byte piece p of row r at r * 128 + ((p ^ (r & 7)) << 4), the
// 128-byte swizzle of the store's tensor map, free of bank conflicts.
__device__ __forceinline__ void stage_row_sw128(uint8_t* block, int r, int chunk, const uint4 (&w)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int p = chunk * 4 + j;
    *reinterpret_cast<uint4*>(block + r * 128 + ((p ^ (r & 7)) << 4)) = w[j];
  }
}

// Expert hidden table: out[row][col] = fp16(gelu_erf(v)) for the expert-
// expansion GEMM E @ W1^T (row = expert id, col = hidden unit; model.py:323
// evaluated once per expert instead of once per selection), stored through
// the tensor map tmC.
struct EpiGeluF16 : EpiNoColParams {
  static constexpr int kEpiWarps = 16;  // 0.117 ms vs 0.126 ms with 8 (262144 x 512 table)
  // The table rows leave through TMA stores of each warp's staged 32 x 64
  // block: written directly, every warp store instruction touched 32 rows
  // with 16-byte pieces and the LSU path bound the kernel (l1tex 79 % busy,
  // 16.8 M L2 write requests per launch).
  static constexpr bool kTmaStore = true;
  __device__ __forceinline__ void operator()(int, int, float (&v)[32], const uint8_t*, const EpiCtx& cx) const {
    uint4 w4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float g0, g1;
        gelu_erf2(v[8 * j + 2 * u], v[8 * j + 2 * u + 1], g0, g1);
        const __half2 hh = __floats2half2_rn(g0, g1);
        w[u] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      w4[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    stage_row_sw128(cx.stg, cx.lane, cx.chunk, w4);
  }
};

// Backward tables: H = fp16(gelu_erf(v)) (tmC) and G = fp16(gelu_erf'(v))
// (tmD) for the pre-activations v = E @ W1^T of every expert, each through
// TMA stores of the warp's staged blocks (H block, then G block 4 KB later).
struct EpiGeluBwdF16 : EpiNoColParams {
  static constexpr int kEpiWarps = 16;
  static constexpr bool kTmaStore = true;
  static constexpr int kTmaOutputs = 2;
  __device__ __forceinline__ void operator()(int, int, float (&v)[32], const uint8_t*, const EpiCtx& cx) const {
    uint4 h4[4], g4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t wh[4], wg[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float ga, gb, da, db;
        gelu_erf_and_grad2(v[8 * j + 2 * u], v[8 * j + 2 * u + 1], ga, gb, da, db);
        const __half2 hh = __floats2half2_rn(ga, gb);
        const __half2 gg = __floats2half2_rn(da, db);
        wh[u] = *reinterpret_cast<const uint32_t*>(&hh);
        wg[u] = *reinterpret_cast<const uint32_t*>(&gg);
      }
      h4[j] = make_uint4(wh[0], wh[1], wh[2], wh[3]);
      g4[j] = make_uint4(wg[0], wg[1], wg[2], wg[3]);
    }
    stage_row_sw128(cx.stg, cx.lane, cx.chunk, h4);
    stage_row_sw128(cx.stg + 32 * 128, cx.lane, cx.chunk, g4);
  }
};

// ---------------------------------------------------------------- kernel --
// Shared-memory descriptor of an MN-major operand in the 128-byte swizzle
// canonical layout: 64-element MN rows of 128 B per K index, 8 K rows per
// 1024-B atom (SBO = 1024), consecutive 64-element MN blocks `lbo` bytes
// apart.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32_major(int M, int N, bool a_mn, bool b_mn) {
  return umma_idesc_bf16_f32(M, N) | (a_mn ? (1u << 15) : 0u) | (b_mn ? (1u << 16) : 0u);
}

template <class Epi, bool kAMN, bool kBMN, int BN>
__global__ void __launch_bounds__(GemmCfg<Epi>::kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD, int M, int N, int K,
           int ksplit, Epi epi, int* err, int hold_unit) {
  static_assert(BN == 128 || BN == 256, "N tile is 128 or 256");
  constexpr int B_BYTES = BN * GEMM_BK * 2;
  constexpr int STAGE_BYTES = GEMM_A_BYTES + B_BYTES;
  using Cfg = GemmCfg<Epi>;
  constexpr int STAGES = Cfg::kStages;
  constexpr int CHUNKS = (BN / 32) / (Cfg::kEpiWarps / 4);  // 32-column chunks per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* colp_s = smem + STAGES * GEMM_STAGE_BYTES;
  uint8_t* stg_s = colp_s + Cfg::kColpBytes;
  GemmCtl* ctl = reinterpret_cast<GemmCtl*>(stg_s + Cfg::kEpiWarps * Cfg::kStgWarpBytes);
  static_assert(!Epi::kTmaStore || CHUNKS == 2, "a TMA-store epilogue stages two 32-column chunks per warp");
  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  const int kpb = (num_kb + ksplit - 1) / ksplit;  // K blocks per split (host guarantees none is empty)
  const int num_units = num_tiles * ksplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], Cfg::kEpiThreads);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  pdl_launch_dependents();
  pdl_wait();  // set-up above touched only shared memory, TMEM and parameters
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      RingPos rp;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
        const int tile = u % num_tiles;
        const int ks = u / num_tiles;
        const int m0 = (tile / num_n) * GEMM_BM;
        const int n0 = (tile % num_n) * BN;
        const int kb1 = min(num_kb, (ks + 1) * kpb);
        if (u == hold_unit) {
          // failure-detection test hook (ethos_test_gemm_withhold; -1 on
          // every production launch): this unit's operands are never
          // loaded, so the MMA issuer's bounded wait for them runs out
          ok = false;
          break;
        }
        for (int kb = ks * kpb; kb < kb1; ++kb) {
          if (!mbar_wait(&ctl->empty[rp.stage], rp.phase ^ 1u, abort, err, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + rp.stage * GEMM_STAGE_BYTES;
          uint8_t* sb = sa + GEMM_A_BYTES;
          mbar_arrive_expect_tx(&ctl->full[rp.stage], STAGE_BYTES);
          if (kAMN) {
            tma_load_2d(sa, &tmA, &ctl->full[rp.stage], m0, kb * GEMM_BK);
            tma_load_2d(sa + 8192, &tmA, &ctl->full[rp.stage], m0 + 64, kb * GEMM_BK);
          } else {
            tma_load_2d(sa, &tmA, &ctl->full[rp.stage], kb * GEMM_BK, m0);
          }
          if (kBMN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 8192, &tmB, &ctl->full[rp.stage], n0 + 64 * j, kb * GEMM_BK);
          } else {
            tma_load_2d(sb, &tmB, &ctl->full[rp.stage], kb * GEMM_BK, n0);
          }
          rp.advance(STAGES);
        }
      }
      if (!ok) rp.drain(ctl->full, STAGES, err, 5);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32_major(GEMM_BM, BN, kAMN, kBMN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;  // false once this role gave up (abort or timeout)
      for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x, ++it) {
        const int ks = u / num_tiles;
        const int kb0 = ks * kpb, kb1 = min(num_kb, (ks + 1) * kpb);
        const int buf = it & 1;
        const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
        if (!mbar_wait(&ctl->acc_empty[buf], acc_phase ^ 1u, abort, err, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort, err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * GEMM_STAGE_BYTES);
          const uint32_t b_base = a_base + GEMM_A_BYTES;
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            const uint64_t ad = kAMN ? umma_desc_sw128_mn(a_base + k * 2048, 8192) : umma_desc_sw128(a_base + k * 32);
            const uint64_t bd = kBMN ? umma_desc_sw128_mn(b_base + k * 2048, 8192) : umma_desc_sw128(b_base + k * 32);
            umma_bf16(d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&ctl->empty[stage]);
          if (++stage == STAGES) {
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
    // Epilogue warps never leave the unit loop early: after an abort they skip
    // the work but still take every named barrier, so no partner can block.
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;  // column group of the tile (CHUNKS chunks each)
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      const int tile = u % num_tiles;
      const int buf = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
      const int m0 = (tile / num_n) * GEMM_BM;
      const int n0 = (tile % num_n) * BN;
      uint8_t* cps = colp_s + buf * 256 * 8;
      if (Epi::kColParamBytes > 0) {
        // stage this tile's column data (its previous user, unit it-2, was
        // released by the barrier of unit it-1)
        const int tid = static_cast<int>(threadIdx.x) - 64;
        if (tid < 256) epi.load_col_params(n0, cps, tid);
        named_bar_sync(1, Cfg::kEpiThreads);
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&ctl->acc_full[buf], acc_phase, abort, err, 4));
      if (!ok) continue;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      EpiCtx cx{stg_s + (warp - 2) * Cfg::kStgWarpBytes, m0 + q * 32, min(32, M - (m0 + q * 32)), lane, 0};
      if constexpr (Epi::kTmaStore) {
        // the previous tile's store must be done reading the staging block
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
      }
#pragma unroll 1
      for (int c = ch * CHUNKS; c < (ch + 1) * CHUNKS; ++c) {
        float v[32];
        tmem_ld32(tmem_addr(tmem, q * 32, buf * BN + c * 32), v);
        cx.chunk = c - ch * CHUNKS;
        epi(row, n0 + c * 32, v, cps, cx);
      }
      tc_fence_before();
      mbar_arrive(&ctl->acc_empty[buf]);
      if constexpr (Epi::kTmaStore) {
        fence_proxy_async_smem();  // the lanes' staging writes, visible to the TMA unit
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, cx.stg, n0 + ch * CHUNKS * 32, m0 + q * 32);
          if constexpr (Cfg::kTmaOutputs == 2) tma_store_2d(&tmD, cx.stg + 32 * 128, n0 + ch * CHUNKS * 32, m0 + q * 32);
          bulk_commit();
        }
      }
    }
    // the CTA's shared memory must outlive the stores' reads, and the table
    // is complete when the kernel ends
    if constexpr (Epi::kTmaStore) {
      if (lane == 0) bulk_wait<0>();
    }
  }

  // Teardown: on the normal path the epilogue consumed every committed
  // accumulator; on the abort path the producer and the MMA issuer drained
  // their in-flight copies and MMAs above.
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

}  // namespace ethos
