// sm_100a building blocks: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (UMMA) descriptors / MMA issue / commit, and TMEM alloc, load, store.
//
// Every wait in this library is bounded: a wait that exceeds the wait limit
// (g_wait_limit_ns, kWaitLimitNs unless ethos_set_wait_limit_ns changed it; or
// sees the CTA's abort flag) records an error code in the caller's global error
// word and returns false, and the kernels then drain and free TMEM before they
// return.  Nothing here traps.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ethos_b200.h"

namespace ethos {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: no legitimate wait comes close

// Per-device wait limit read by mbar_wait once it starts checking the clock
// (ethos_set_wait_limit_ns; a test shortens it to make a withheld stage time
// out quickly).  Only the slow path of a wait reads it.
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Records the first error code of a launch (later ones are dropped).
__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------ dependent launches --
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream is still
// running.  pdl_launch_dependents() lets the next kernel start launching;
// pdl_wait() blocks until the previous kernel has completed and its memory
// is visible, and must come before this kernel's first global-memory access.
// Both are no-ops for a kernel launched the ordinary way.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  `abort` is a CTA-shared
// flag: once any role gives up, every other wait returns false promptly.  A
// null `abort` makes a drain wait (used on the abort path itself): it only
// ends on completion or on the time limit.
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                       int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  const uint64_t limit = *static_cast<volatile unsigned long long*>(&g_wait_limit_ns);
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (abort != nullptr && *abort) return false;
      if (global_timer_ns() - t0 > limit) {
        if (abort != nullptr) *abort = 1;
        record_error(err, ETHOS_ERR_TIMEOUT_BASE + site);
        return false;
      }
    }
  }
}

// Producer-side ring position with drain support: after an abort, waits for
// the `full` phases of the (up to `stages`) most recent loads still in flight
// so that no bulk copy lands in shared memory after the CTA exits.
struct RingPos {
  int stage = 0;
  uint32_t phase = 0;
  int issued = 0;
  __device__ __forceinline__ void advance(int stages) {
    ++issued;
    if (++stage == stages) {
      stage = 0;
      phase ^= 1u;
    }
  }
  __device__ void drain(uint64_t* full, int stages, int* err, int site) const {
    int s = stage;
    uint32_t ph = phase;
    for (int i = 0; i < stages && i < issued; ++i) {
      if (s == 0) {
        s = stages - 1;
        ph ^= 1u;
      } else {
        --s;
      }
      mbar_wait(&full[s], ph, nullptr, err, site);
    }
  }
};

// --------------------------------------------------------------------- TMA --
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared (no multicast), completion
// counted in bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tm, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Make generic-proxy writes to shared memory visible to the async proxy
// (tcgen05.mma operand reads, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2-D tiled bulk tensor store shared -> global (this GPU's memory), tracked
// by the issuing thread's bulk groups.  The box's rows outside the tensor are
// not written.  x (the contiguous coordinate) must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N of this thread's bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until at most N of this thread's bulk groups are incomplete (writes done)
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------ cp.async 16B --
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------- named barriers --
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------- UMMA descriptors --
// Shared-memory matrix descriptor for a K-major operand stored in the 128-byte
// swizzle canonical layout: rows of 128 B (64 bf16), 8-row groups 1024 B apart
// (stride byte offset), 16-byte chunks XOR-permuted by (row % 8).  Bits:
// [0,14) start>>4, [16,30) leading byte offset>>4 (unused for swizzled K-major,
// set to 1), [32,46) stride byte offset>>4, [46,48) version = 1 (sm_100),
// [61,64) layout = 2 (SWIZZLE_128B).  The tile base must be 1024-B aligned;
// stepping K inside the 128-B atom adds (k_bytes >> 4) to the start field.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// The same for the 64-byte swizzle: rows of 64 B (32 bf16), 8-row groups 512 B
// apart, 16-byte chunks XOR-permuted by (row / 2) % 4; layout = 4
// (SWIZZLE_64B), tile base 512-B aligned, K steps inside the 64-B atom again
// add (k_bytes >> 4) to the start field.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;
  return d;
}

// And for the 32-byte swizzle: rows of 32 B (16 bf16, one K step), 8-row
// groups 256 B apart, layout = 6 (SWIZZLE_32B), tile base 256-B aligned.
__device__ __forceinline__ uint64_t umma_desc_sw32(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(256u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(6u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major.
// Bits: [4,6) D format (1 = f32), [7,10) A format (1 = bf16), [10,13) B format
// (1 = bf16), bit 15/16 A/B major (0 = K), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ----------------------------------------------------------------- tcgen05 --
__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Warp-collective: each lane reads 32 consecutive fp32 columns of its TMEM lane
// (lane quarter = warp % 4).  The wait is fused so the registers are valid on
// return.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive fp32 columns per lane: two loads in flight, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]),
        "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]),
        "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]),
        "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
        "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr), "r"(taddr + 32u)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp-collective store of 32 fp32 columns per lane; completion is awaited by
// tmem_wait_st() before the same columns are read again.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// TMEM address of (lane, column).
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ------------------------------------------------------------------- math --
// Packed fp32 pairs (sm_100 f32x2 arithmetic): one 64-bit register pair
// holds two floats, fma.rn.f32x2 does two FMAs per instruction.
__device__ __forceinline__ unsigned long long pk2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ unsigned long long fmul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float ex2_approx(float t) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
  return r;
}

// The erf-form GELU, GELU(x) = x Phi(x) (torch.nn.functional.gelu with
// approximate='none'), with the normal CDF written through its tail mass
//   h = 1 - Phi(|x|) = 0.5 exp(-x^2 / 2) erfcx(|x| / sqrt(2)):
//   Phi(x) = 1 - h (x >= 0),  Phi(x) = h (x < 0),  GELU(x) = max(x, 0) - |x| h.
// h is one power of two, h = 2^(kE x^2 + Q(u)), kE = -1 / (2 ln 2), where
// Q(a) = log2(0.5 erfcx(a / sqrt 2)) is a degree-7 polynomial in
// u = min(|x|, kA) * (2 / kA) - 1 fitted by weighted minimax (Lawson's
// algorithm; csrc/fit_gelu.py): fp32 evaluation within 1.9e-7 of Phi and
// 7.1e-8 + 2^-23 |GELU| of the erf GELU.  Clamping |x| at kA = 5.5 keeps the
// Gaussian factor exact, so the tail stays below the true mass times
// |x| / 5.5 there.  One ex2.approx per value and no reciprocal; the
// derivative d GELU / dx = Phi(x) + x phi(x) takes the density from a second
// one, phi(x) = 2^(kE x^2 + log2(1 / sqrt(2 pi))).
namespace gelu_detail {
constexpr float kA = 5.500000000e+00f;    // clamp of |x| for the polynomial
constexpr float kU = 3.636363745e-01f;    // 2 / kA: u = min(|x|, kA) kU - 1
constexpr float kE = -7.213475108e-01f;   // -1 / (2 ln 2): exp(-x^2 / 2) = 2^(kE x^2)
constexpr float kPdf2 = -1.325748086e+00f;  // log2(1 / sqrt(2 pi))
constexpr float Q0 = -2.935396671e+00f, Q1 = -1.197389245e+00f, Q2 = 4.303870797e-01f, Q3 = -1.840556413e-01f,
                Q4 = 8.516710997e-02f, Q5 = -8.533163927e-03f, Q6 = 3.714597598e-02f, Q7 = 7.281220052e-03f;
}  // namespace gelu_detail

// exponent of h = 2^(kE x^2 + Q(u)) for one value
__device__ __forceinline__ float gelu_tail_exponent(float x) {
  using namespace gelu_detail;
  const float u = fmaf(fminf(fabsf(x), kA), kU, -1.0f);
  float q = Q7;
  q = fmaf(q, u, Q6);
  q = fmaf(q, u, Q5);
  q = fmaf(q, u, Q4);
  q = fmaf(q, u, Q3);
  q = fmaf(q, u, Q2);
  q = fmaf(q, u, Q1);
  q = fmaf(q, u, Q0);
  return fmaf(x * x, kE, q);
}

// h = 1 - Phi(|x|) for two values, the polynomial and the exponent on packed
// pairs (the same fp32 operations as the scalar form, so the same results)
__device__ __forceinline__ void gelu_tail2(float x0, float x1, float& h0, float& h1) {
  using namespace gelu_detail;
  const unsigned long long u = ffma2(pk2(fminf(fabsf(x0), kA), fminf(fabsf(x1), kA)), pk2(kU, kU), pk2(-1.0f, -1.0f));
  unsigned long long q = pk2(Q7, Q7);
  q = ffma2(q, u, pk2(Q6, Q6));
  q = ffma2(q, u, pk2(Q5, Q5));
  q = ffma2(q, u, pk2(Q4, Q4));
  q = ffma2(q, u, pk2(Q3, Q3));
  q = ffma2(q, u, pk2(Q2, Q2));
  q = ffma2(q, u, pk2(Q1, Q1));
  q = ffma2(q, u, pk2(Q0, Q0));
  const unsigned long long xv = pk2(x0, x1);
  const unsigned long long s = ffma2(fmul2(xv, xv), pk2(kE, kE), q);
  float s0, s1;
  upk2(s, s0, s1);
  h0 = ex2_approx(s0);
  h1 = ex2_approx(s1);
}
__device__ __forceinline__ float gelu_tail(float x) { return ex2_approx(gelu_tail_exponent(x)); }
__device__ __forceinline__ float gelu_erf(float x) { return fmaf(-fabsf(x), gelu_tail(x), fmaxf(x, 0.0f)); }
// normal density phi(x) = 2^(kE x^2 + log2(1 / sqrt(2 pi)))
__device__ __forceinline__ float gelu_pdf(float x) {
  return ex2_approx(fmaf(x * x, gelu_detail::kE, gelu_detail::kPdf2));
}
// d GELU / dx = Phi(x) + x phi(x)
__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float h = gelu_tail(x);
  const float phi = x >= 0.0f ? 1.0f - h : h;
  return fmaf(x, gelu_pdf(x), phi);
}
__device__ __forceinline__ void gelu_erf2(float x0, float x1, float& g0, float& g1) {
  float h0, h1;
  gelu_tail2(x0, x1, h0, h1);
  g0 = fmaf(-fabsf(x0), h0, fmaxf(x0, 0.0f));
  g1 = fmaf(-fabsf(x1), h1, fmaxf(x1, 0.0f));
}
// GELU and its derivative of two values from one tail evaluation
__device__ __forceinline__ void gelu_erf_and_grad2(float x0, float x1, float& g0, float& g1, float& d0, float& d1) {
  float h0, h1;
  gelu_tail2(x0, x1, h0, h1);
  g0 = fmaf(-fabsf(x0), h0, fmaxf(x0, 0.0f));
  g1 = fmaf(-fabsf(x1), h1, fmaxf(x1, 0.0f));
  const float p0 = x0 >= 0.0f ? 1.0f - h0 : h0, p1 = x1 >= 0.0f ? 1.0f - h1 : h1;
  d0 = fmaf(x0, gelu_pdf(x0), p0);
  d1 = fmaf(x1, gelu_pdf(x1), p1);
}

// Warp transpose-reduce: on entry lane l holds v[0..31] (32 columns of one
// row); on return lane l holds the sum over all 32 lanes of column l.
__device__ __forceinline__ float warp_transpose_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? v[i] : v[i + w];
      const float keep = up ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return __shfl_sync(0xffffffffu, threadIdx.x >> 5, 0); }

}  // namespace ethos
