// sm_100a building blocks shared by every tensor-core kernel in abacus_b200:
// mbarriers with bounded waits, TMA tile loads (no cluster multicast anywhere),
// tcgen05 TMEM allocation / MMA / commit / load, and UMMA descriptors.
//
// Descriptor bit layouts follow the PTX ISA "tcgen05 matrix descriptors" and
// "instruction descriptor" tables (the same fields CUTLASS names in
// cute/arch/mma_sm100_desc.hpp).
//
// Every wait in this file is bounded: after ABACUS_WAIT_NS of %globaltimer
// time it records an error code in the caller's status word and returns
// false, so a kernel whose producer died never spins forever.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifndef ABACUS_WAIT_NS
#define ABACUS_WAIT_NS 2000000000ull  // 2 s per wait
#endif
// Waits on another GPU's progress (its kernels may legitimately run a whole
// layer behind) use a longer bound.
#ifndef ABACUS_PEER_WAIT_NS
#define ABACUS_PEER_WAIT_NS 30000000000ull  // 30 s
#endif

namespace abacus {

// Error codes written to the device status word.
enum : int {
  kStatusOk = 0,
  kStatusTimeoutFull = 1,     // consumer waited for a TMA stage that never landed
  kStatusTimeoutEmpty = 2,    // producer waited for a stage the MMA never released
  kStatusTimeoutAccum = 3,    // epilogue waited for an accumulator that never completed
  kStatusTimeoutConvert = 4,  // MMA waited for the split-precision converter
  kStatusTimeoutPeer = 5,     // waited for a peer GPU's flag
  kStatusBadArgs = 6,
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n"
      ".reg .pred P;\n"
      "elect.sync _|P, 0xffffffff;\n"
      "selp.b32 %0, 1, 0, P;\n"
      "}\n"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred P;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n"
      "selp.b32 %0, 1, 0, P;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false (and records `code` in *status) on timeout, or
// immediately if another CTA already recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t iter = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++iter & 255u) == 0) {
      if (status != nullptr && *reinterpret_cast<volatile int*>(status) != kStatusOk) return false;
      if (globaltimer_ns() - start > ABACUS_WAIT_NS) {
        if (status != nullptr) atomicCAS(status, kStatusOk, code);
        return false;
      }
    }
  }
}

// Warp-uniform bounded wait for roles where all 32 lanes wait and then issue
// warp-collective (.sync.aligned) tcgen05 instructions: the result is the same
// on every lane, so a timeout can never split the warp around such an op.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* status, int code) {
  const bool ok = mbar_wait(bar, parity, status, code);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------- register split
// Per-warpgroup register budgets (all four warps of a warpgroup execute it).
// The increases draw on what the decreases of the other warpgroups give
// back, within the registers the block was launched with.
template <uint32_t N>
__device__ __forceinline__ void regs_increase() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_decrease() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- CTA pairs
// Two CTAs of a (2, 1, 1) cluster on neighbouring SMs share one tcgen05 MMA
// (cta_group::2): each holds half of A's rows (and of D) and half of B's
// columns, so every SM reads only its half of B from its own shared memory.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// Arrive on a barrier of any CTA of the cluster (default semantics: release
// at CTA scope; a release at cluster scope costs a memory barrier per arrive
// (measured: membar stalls took the pair GEMM below the single-CTA one). The
// data the arrive publishes is ordered by the async-proxy fences the callers
// issue first: fence.proxy.async for shared-memory writes and
// tcgen05.wait::st + tcgen05.fence::before_thread_sync for TMEM.)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// All threads of both CTAs (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- peer flags
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *flag >= target (signed compare of monotonic counters
// that another GPU advances). On timeout records kStatusTimeoutPeer.
__device__ __forceinline__ bool wait_flag_geq(const int* flag, int target, int* status) {
  if (ld_acquire_sys(flag) - target >= 0) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t iter = 0;
  while (true) {
    __nanosleep(64);
    if (ld_acquire_sys(flag) - target >= 0) return true;
    if ((++iter & 63u) == 0) {
      if (status != nullptr && *reinterpret_cast<volatile int*>(status) != kStatusOk) return false;
      if (globaltimer_ns() - start > ABACUS_PEER_WAIT_NS) {
        if (status != nullptr) atomicCAS(status, kStatusOk, kStatusTimeoutPeer);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled load global -> shared, completion counted on `bar` in bytes.
// Coordinates: x is the innermost (contiguous) dimension in elements.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled load (x innermost).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// ---------------------------------------------------------------- TMEM
// Allocation is a warp-wide operation; the allocated base address is written
// to `dst_smem`. ncols must be a power of two >= 32.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Pair TMEM allocation: one warp of EACH CTA of the pair issues it (same
// warp index, same shared-memory slot); both receive the same address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Pair MMA, kind::tf32, issued by one thread of the even CTA: D (both CTAs'
// TMEM, 128 lanes each) (+)= A (both CTAs' TMEM at a_tmem) * B (both CTAs'
// shared memory at the descriptor's offset: columns [0, N/2) in the even CTA,
// [N/2, N) in the odd one).
__device__ __forceinline__ void mma_tf32_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// Arrive once on the barrier at `cluster_addr` (this CTA's or the peer's,
// from mapa_shared) when every pair MMA issued so far by this thread is done.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

// D(tmem) (+)= A(smem) * B(smem), kind::tf32, issued by a single thread.
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem), kind::tf32. A is K-major in TMEM: lane = row
// of A, one 32-bit column per K element.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive once on `bar` when every MMA previously issued by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its own TMEM
// lane. The warp may only touch lanes [32*(warp%4), 32*(warp%4)+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Each thread writes 32 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05, "version 1").
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 version = 1
//   bits 49-51 base offset (0: every buffer here is aligned to its swizzle period)
//   bit  52    LBO mode (0)
//   bits 61-63 layout: 0 none, 1 128B with 32B atoms, 2 128B, 4 64B, 6 32B
enum : uint32_t { kLayoutSw128Base32 = 1, kLayoutSw128 = 2 };

__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// K-major operand tile: rows of 128 bytes (32 fp32 along K), 8-row swizzle
// atoms of 1024 bytes, loaded by TMA with SWIZZLE_128B.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
  return make_smem_desc(saddr, 16, 1024, kLayoutSw128);
}

// MN-major 32-bit operand tile: chunks of 32 elements along M/N (128 bytes) x
// `rows` K-rows, chunk stride `chunk_bytes`; 32-byte granules swizzled with a
// period of 4 rows (TMA SWIZZLE_128B_ATOM_32B).
__device__ __forceinline__ uint64_t desc_mnmajor_sw128_32b(uint32_t saddr, uint32_t chunk_bytes) {
  return make_smem_desc(saddr, chunk_bytes, 512, kLayoutSw128Base32);
}

// Instruction descriptor for kind::tf32 with an fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                  // D format f32
         | (2u << 7)                                // A format tf32
         | (2u << 10)                               // B format tf32
         | ((a_mn_major ? 1u : 0u) << 15)           // A major
         | ((b_mn_major ? 1u : 0u) << 16)           // B major
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// Split-precision helper (3xTF32, Markidis et al. 2018 / Ootomo & Yokota 2022):
// x = hi + lo with hi, lo both representable in tf32.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// The same rounding (to nearest, ties away from zero, onto 10 explicit
// mantissa bits) on the integer ALUs: adding half a tf32 ulp (bit 12) to the
// magnitude bits carries into bit 13 exactly when the 13 dropped bits are at
// least half an ulp (a carry out of the mantissa bumps the exponent, which is
// the correctly rounded value), then the dropped bits are cleared. Infinities
// and NaNs (all exponent bits set) pass through unchanged. Used in the
// attention softmax loops, where the conversion would otherwise queue behind
// the exponentials; measured slower than the conversion instruction in the
// GEMM split converter, which therefore keeps to_tf32.
__device__ __forceinline__ float to_tf32_alu(float x) {
  const uint32_t u = __float_as_uint(x);
  const uint32_t r = (u + 0x1000u) & 0xffffe000u;
  return __uint_as_float((u & 0x7f800000u) == 0x7f800000u ? u : r);
}

// The low part of a split, lo = x - hi, rounded the same way but without the
// Inf / NaN pass-through: when x is Inf or NaN, hi already carries it into the
// product, so the value of lo does not matter. Two integer operations.
__device__ __forceinline__ float to_tf32_lo(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
}

// hi part on the conversion unit and lo on the integer ALUs: the two
// halves of a softmax-loop split run on different pipes.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = to_tf32(x);
  lo = to_tf32_lo(x - hi);
}

// 2^x on the special-function unit (ex2.approx, denormal results flushed to
// zero). Softmax probabilities below 2^-126 are zero for training purposes.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The value a kind::tf32 MMA uses for an fp32 operand element read from shared
// memory or TMEM: the low 13 mantissa bits dropped (measured on B200). An
// operand left as raw fp32 therefore acts as its own "hi" part, and only
// lo = tf32(x - tf32_trunc(x)) must be written beside it.
__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }
__device__ __forceinline__ float tf32_lo_of_raw(float x) { return to_tf32(x - tf32_trunc(x)); }
// The same with the rounding on the integer ALUs (keeps the conversion unit,
// which the GEMM converter also needs for every A element, free).
__device__ __forceinline__ float tf32_lo_of_raw_alu(float x) { return to_tf32_lo(x - tf32_trunc(x)); }

}  // namespace abacus
