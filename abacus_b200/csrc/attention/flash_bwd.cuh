// Causal flash-attention backward on tcgen05 (kind::tf32), fp32 in / out.
//
// Two deterministic kernels (no atomics), each recomputing the scores of its
// tiles from Q, K and the forward's log-sum-exp:
//
//   flash_bwd_dkdv: one CTA = 128 keys of one (batch, head); visits the query
//     blocks that can see those keys.
//        S^T  = K Q_i^T,  dP^T = V dO_i^T            (smem A and B, K-major)
//        P^T  = exp(S^T * scale - lse),  dS^T = P^T (dP^T - Delta)   (threads)
//        dV  += P^T dO_i,  dK += dS^T Q_i             (A = TMEM, B MN-major)
//   flash_bwd_dq: one CTA = 128 queries; visits the visible key blocks.
//        S = Q K_j^T, dP = dO V_j^T  ->  dS  ->  dQ += dS K_j
//
// tf32 operands cannot share one shared-memory tile between a K-major and an
// MN-major read (the MN-major 32-bit layout uses its own swizzle), so tiles
// used both ways are loaded twice by TMA, once per layout.
//
// Accumulation precision: in 3xTF32 mode every per-block partial (dV, dK,
// dQ) lands in a fresh TMEM buffer and is added with round-to-nearest fp32
// adds by the threads (into TMEM masters for dK/dV, registers for dQ).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cfloat>
#include <climits>
#include <cstdint>
#include "../common/sm100.cuh"

namespace abacus {
namespace attn {

struct BwdParams {
  // dkdv kernel: K / V tiles (128 rows, K-major), Q and dO tiles (inner block,
  // K-major and MN-major). dq kernel: Q / dO (128 rows, K-major), K_j (K-major
  // and MN-major), V_j (K-major).
  CUtensorMap tma_q_k, tma_q_mn, tma_do_k, tma_do_mn;
  CUtensorMap tma_k_k, tma_k_mn, tma_v_k;
  const float* lse;    // (B, H, Lq), natural log of the scaled scores
  const float* delta;  // (B, H, Lq), rowsum(dO * O)
  float* dq;           // (B*Lq, ld_dq)
  long long ld_dq;
  float* dk;           // (B*Lk, ld_dk)
  long long ld_dk;
  float* dv;
  long long ld_dv;
  const int64_t* q_pos;
  const int64_t* k_pos;
  int batch, heads, lq, lk;
  float scale;         // softmax scale
  float scale_log2;    // scale * log2(e)
  // Context parallel: dK / dV rows of the gathered keys go to their owner's
  // staging slot (row (b*lk + k) -> owner k / chunk, local row b*chunk +
  // k % chunk, row stride ld_dk / ld_dv) and each finished 128-key tile adds
  // 1 to the owner's arrival counter (scatter_chunk 0: plain stores).
  float* scatter_dk[8];
  float* scatter_dv[8];
  unsigned* scatter_counter[8];
  int scatter_chunk;
  int* status;
  // Optional phase trace of the dK/dV kernel (clock64 stamps of CTA (0, 0, 0),
  // slot * 64 + block): 0 S^T / dP^T issued, 1 S^T seen by the threads,
  // 2 P^T / dS^T written, 3 dV / dK issued, 4 partials drained, 5 K-major
  // tiles split, 6 MN-major tiles split, 7 K-major load issued, 8 MN-major
  // load issued.
  long long* trace;
};

constexpr float kLog2e = 1.4426950408889634f;

// Visible inner blocks of an outer tile, with a "needs masking" flag.
// outer_is_query: the outer tile holds queries (dq kernel) or keys (dkdv).
template <int OUTER, int INNER, int MAXB>
__device__ void build_block_list(const BwdParams& p, bool outer_is_query, int o0, int* list, int* n_out, int lane) {
  const int outer_len = outer_is_query ? p.lq : p.lk;
  const int inner_len = outer_is_query ? p.lk : p.lq;
  const int64_t* opos = outer_is_query ? p.q_pos : p.k_pos;
  const int64_t* ipos = outer_is_query ? p.k_pos : p.q_pos;
  int omin = INT_MAX, omax = INT_MIN;
  for (int i = lane; i < OUTER; i += 32) {
    const int oi = o0 + i;
    if (oi < outer_len) {
      const int pos = opos ? static_cast<int>(opos[oi]) : oi;
      omin = min(omin, pos);
      omax = max(omax, pos);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    omin = min(omin, __shfl_xor_sync(0xffffffffu, omin, o));
    omax = max(omax, __shfl_xor_sync(0xffffffffu, omax, o));
  }
  const int nib = (inner_len + INNER - 1) / INNER;
  int count = 0;
  for (int base = 0; base < nib; base += 32) {
    const int ib = base + lane;
    bool keep = false, partial = false;
    if (ib < nib) {
      int imin = INT_MAX, imax = INT_MIN;
      for (int i = 0; i < INNER; ++i) {
        const int ii = ib * INNER + i;
        if (ii < inner_len) {
          const int pos = ipos ? static_cast<int>(ipos[ii]) : ii;
          imin = min(imin, pos);
          imax = max(imax, pos);
        }
      }
      if (outer_is_query) {  // inner = keys: visible if some key <= some query
        keep = imin <= omax;
        partial = imax > omin;
      } else {  // inner = queries: visible if some query >= some key
        keep = imax >= omin;
        partial = imin < omax;
      }
      partial = partial || (ib * INNER + INNER > inner_len) || (o0 + OUTER > outer_len);
    }
    const unsigned mask = __ballot_sync(0xffffffffu, keep);
    if (keep) {
      const int slot = count + __popc(mask & ((1u << lane) - 1u));
      if (slot < MAXB) list[slot] = ib | (partial ? (1 << 30) : 0);
    }
    count += __popc(mask);
  }
  if (lane == 0) {
    *n_out = min(count, MAXB);
    if (count > MAXB) atomicCAS(p.status, kStatusOk, kStatusBadArgs);
  }
}

__device__ __forceinline__ void split_tile(uint8_t* hi_buf, uint8_t* lo_buf, int bytes, int tid, int nthreads) {
  float4* hi = reinterpret_cast<float4*>(hi_buf);
  float4* lo = reinterpret_cast<float4*>(lo_buf);
  for (int i = tid; i < bytes / 16; i += nthreads) {
    // hi stays raw (the MMA truncates it to tf32); only lo is written.
    const float4 x = hi[i];
    lo[i] = make_float4(tf32_lo_of_raw(x.x), tf32_lo_of_raw(x.y), tf32_lo_of_raw(x.z), tf32_lo_of_raw(x.w));
  }
}

// ============================================================================ dK / dV
template <int D, int PASSES>
struct DkdvCfg {
  static constexpr int kOuter = 128;                     // keys per CTA
  static constexpr int kInner = (PASSES == 3 || D == 128) ? 32 : 64;  // queries per block
  static constexpr int kSplit = PASSES == 3 ? 2 : 1;
  static constexpr int kKVTile = kOuter * D * 4;         // K or V
  static constexpr int kQTile = kInner * D * 4;          // one layout of Q or dO
  static constexpr int kStageBytes = 4 * kQTile * kSplit;  // Q_k, Q_mn, dO_k, dO_mn [+ lo]
  static constexpr int kSmemRaw = 2 * kKVTile * kSplit + kStageBytes + 1024;
  static constexpr int kThreads = PASSES == 3 ? 320 : 192;
  // Register cap for one CTA per SM: each of the 4 SM sub-partitions holds
  // 16384 registers and ceil(warps / 4) of the CTA's warps.
  static constexpr int kWarpsPerSubpartition = (kThreads / 32 + 3) / 4;
  static constexpr int kMaxRegs =
      (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8 > 255 ? 255 : (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8;
  // TMEM: two buffers (blocks alternate) of ST (S^T, P^T hi [, P^T lo]) and
  // DPT (dP^T, dS^T hi [, dS^T lo]), so the next block's score MMAs run while
  // the threads turn this block's scores into P^T / dS^T; then the dV, dK
  // partials [+ dV, dK masters in 3xTF32 mode].
  static constexpr int kSTCols = kInner * kSplit;
  static constexpr int kST = 0, kDPT = kSTCols, kBufCols = 2 * kSTCols;
  static constexpr int kDVp = 2 * kBufCols, kDKp = kDVp + D;
  static constexpr int kDVm = kDKp + D, kDKm = kDVm + D;
  static constexpr int kCols = PASSES == 3 ? kDKm + D : kDKp + D;
  static constexpr uint32_t kTmemCols = kCols <= 256 ? 256 : 512;
  static constexpr int kMaxBlocks = 2048;
  // A CTA that takes all 512 TMEM columns must be alone on its SM (a second
  // one would wait in tcgen05.alloc for the first to finish): ask for more
  // than half of the SM's shared memory.
  static constexpr int kSmemBytes = (kTmemCols == 512 && kSmemRaw < 116 * 1024) ? 116 * 1024 : kSmemRaw;
};

template <int D, int PASSES>
__global__ void __maxnreg__((DkdvCfg<D, PASSES>::kMaxRegs)) flash_bwd_dkdv_kernel(const __grid_constant__ BwdParams p) {
  using Cfg = DkdvCfg<D, PASSES>;
  constexpr int NQ = Cfg::kInner;
  static_assert(Cfg::kCols <= 512, "TMEM budget");
  extern __shared__ uint8_t smem_raw[];
  // Q / dO tiles come in two groups with their own barriers: the K-major
  // tiles (S^T, dP^T MMAs) and the MN-major tiles (dV, dK MMAs), so the next
  // block's K-major tiles load while this block's threads and dV / dK MMAs run.
  __shared__ uint64_t kv_full, kv_conv, st_full[2], p_full[2], part_full;
  __shared__ uint64_t kf_full, kf_conv, kf_empty, mn_full, mn_conv, mn_empty;
  __shared__ uint32_t tmem_slot;
  __shared__ int n_blocks;
  __shared__ int abort_flag;
  __shared__ int block_list[Cfg::kMaxBlocks];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool traced = p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
#define ABACUS_BWD_TRACE(slot, i) \
  if (traced && (i) < 64) p.trace[(slot) * 64 + (i)] = clock64();
  if (threadIdx.x == 0) abort_flag = *reinterpret_cast<volatile int*>(p.status);
  __syncthreads();
  if (abort_flag != kStatusOk) return;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sk = smem;                                   // K hi [, K lo]
  uint8_t* sv = smem + Cfg::kKVTile * Cfg::kSplit;      // V hi [, V lo]
  uint8_t* st = sv + Cfg::kKVTile * Cfg::kSplit;        // Q_k, Q_mn, dO_k, dO_mn, then lo copies
  auto tile = [&](int which, int lo) { return st + (lo * 4 + which) * Cfg::kQTile; };

  const int nkb = (p.lk + 127) / 128;
  (void)nkb;
  const int kb = blockIdx.x;  // early keys see the most queries: schedule them first
  const int h = blockIdx.y, b = blockIdx.z;
  const int k0 = kb * 128;
  const int k_row0 = b * p.lk + k0;
  const int q_row_base = b * p.lq;
  const int col0 = h * D;

  if (threadIdx.x == 0) {
    mbar_init(&kv_full, 1);
    mbar_init(&kv_conv, 128);
    mbar_init(&st_full[0], 1);
    mbar_init(&st_full[1], 1);
    mbar_init(&p_full[0], 128);
    mbar_init(&p_full[1], 128);
    mbar_init(&part_full, 1);
    mbar_init(&kf_full, 1);
    mbar_init(&kf_conv, 128);
    mbar_init(&kf_empty, 1);
    mbar_init(&mn_full, 1);
    mbar_init(&mn_conv, 128);
    mbar_init(&mn_empty, 1);
    fence_mbar_init();
  }
  if (warp == 0) build_block_list<128, NQ, Cfg::kMaxBlocks>(p, false, k0, block_list, &n_blocks, lane);
  if (warp == 1) {
    tmem_alloc(&tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int nb = n_blocks;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(&kv_full, 2 * Cfg::kKVTile);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        tma_load_2d(sk + c * 128 * 128, &p.tma_k_k, &kv_full, col0 + 32 * c, k_row0);
        tma_load_2d(sv + c * 128 * 128, &p.tma_v_k, &kv_full, col0 + 32 * c, k_row0);
      }
      // The K-major tiles run one block ahead of the MN-major ones: block
      // i+1's score MMAs are issued before block i's gradient MMAs.
      int issued_k = 0, issued_mn = 0;
      for (int step = 0; step <= nb; ++step) {
        if (step < nb) {
          const int qrow = q_row_base + (block_list[step] & 0xFFFF) * NQ;
          // K-major Q / dO: free once the previous block's S^T / dP^T MMAs ran.
          if (step >= 1 && !mbar_wait(&kf_empty, (step - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
          ABACUS_BWD_TRACE(7, step)
          mbar_arrive_expect_tx(&kf_full, 2 * Cfg::kQTile);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_2d(tile(0, 0) + c * NQ * 128, &p.tma_q_k, &kf_full, col0 + 32 * c, qrow);
            tma_load_2d(tile(2, 0) + c * NQ * 128, &p.tma_do_k, &kf_full, col0 + 32 * c, qrow);
          }
          ++issued_k;
        }
        if (step >= 1) {
          const int i = step - 1;
          const int qrow = q_row_base + (block_list[i] & 0xFFFF) * NQ;
          // MN-major Q / dO: free once the previous block's dV / dK MMAs ran.
          if (i >= 1 && !mbar_wait(&mn_empty, (i - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
          ABACUS_BWD_TRACE(8, i)
          mbar_arrive_expect_tx(&mn_full, 2 * Cfg::kQTile);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_2d(tile(1, 0) + c * NQ * 128, &p.tma_q_mn, &mn_full, col0 + 32 * c, qrow);
            tma_load_2d(tile(3, 0) + c * NQ * 128, &p.tma_do_mn, &mn_full, col0 + 32 * c, qrow);
          }
          ++issued_mn;
        }
      }
      mbar_wait(&kv_full, 0, nullptr, 0);
      if (issued_k > 0) mbar_wait(&kf_full, (issued_k - 1) & 1, nullptr, 0);
      if (issued_mn > 0) mbar_wait(&mn_full, (issued_mn - 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = idesc_tf32(128, NQ, false, false);
      constexpr uint32_t idesc_acc = idesc_tf32(128, D, false, true);
      bool ok = mbar_wait(PASSES == 3 ? &kv_conv : &kv_full, 0, p.status, kStatusTimeoutFull);
      // S^T = K Q^T and dP^T = V dO^T of block i into TMEM buffer i & 1.
      auto issue_scores = [&](int i) -> bool {
        if (!mbar_wait(PASSES == 3 ? &kf_conv : &kf_full, i & 1, p.status, kStatusTimeoutFull)) return false;
        tc_fence_after();
        const int buf = (i & 1) * Cfg::kBufCols;
#pragma unroll
        for (int pair = 0; pair < 2; ++pair) {
          const uint32_t a_hi = smem_u32(pair == 0 ? sk : sv);
          const uint32_t b_hi = smem_u32(tile(pair == 0 ? 0 : 2, 0));
          const uint32_t b_lo = smem_u32(tile(pair == 0 ? 0 : 2, 1));
          const uint32_t d = tmem + buf + (pair == 0 ? Cfg::kST : Cfg::kDPT);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint32_t ao = c * 128 * 128 + ks * 32;
              const uint32_t bo = c * NQ * 128 + ks * 32;
              const uint32_t acc = (c | ks) ? 1u : 0u;
              if (PASSES == 3) {
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + Cfg::kKVTile + ao), desc_kmajor_sw128(b_hi + bo), idesc_s, acc);
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + ao), desc_kmajor_sw128(b_lo + bo), idesc_s, 1u);
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + ao), desc_kmajor_sw128(b_hi + bo), idesc_s, 1u);
              } else {
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + ao), desc_kmajor_sw128(b_hi + bo), idesc_s, acc);
              }
            }
          }
        }
        ABACUS_BWD_TRACE(0, i)
        mma_commit(&st_full[i & 1]);
        mma_commit(&kf_empty);
        return true;
      };
      // dV (+)= P^T dO and dK (+)= dS^T Q of block i, A from TMEM buffer i & 1.
      // 3xTF32: the tensor core accumulates two consecutive blocks (a 64-deep
      // reduction, as in the GEMM) before the threads fold the partial into
      // the fp32 masters; tf32: everything accumulates in TMEM.
      auto issue_grads = [&](int i) -> bool {
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, p.status, kStatusTimeoutAccum)) return false;
        if (!mbar_wait(PASSES == 3 ? &mn_conv : &mn_full, i & 1, p.status, kStatusTimeoutFull)) return false;
        tc_fence_after();
        const int buf = (i & 1) * Cfg::kBufCols;
#pragma unroll
        for (int pair = 0; pair < 2; ++pair) {
          const uint32_t a = tmem + buf + (pair == 0 ? Cfg::kST : Cfg::kDPT);
          const uint32_t bh = smem_u32(tile(pair == 0 ? 3 : 1, 0));
          const uint32_t bl = smem_u32(tile(pair == 0 ? 3 : 1, 1));
          const uint32_t d = tmem + (pair == 0 ? Cfg::kDVp : Cfg::kDKp);
#pragma unroll
          for (int ks = 0; ks < NQ / 8; ++ks) {
            const uint64_t vb = desc_mnmajor_sw128_32b(bh + ks * 1024, NQ * 128);
            const uint32_t acc = PASSES == 3 ? ((ks | (i & 1)) ? 1u : 0u) : ((i | ks) ? 1u : 0u);
            if (PASSES == 3) {
              const uint64_t vl = desc_mnmajor_sw128_32b(bl + ks * 1024, NQ * 128);
              mma_tf32_ts(d, a + NQ + ks * 8, vb, idesc_acc, acc);
              mma_tf32_ts(d, a + ks * 8, vl, idesc_acc, 1u);
              mma_tf32_ts(d, a + ks * 8, vb, idesc_acc, 1u);
            } else {
              mma_tf32_ts(d, a + ks * 8, vb, idesc_acc, acc);
            }
          }
        }
        ABACUS_BWD_TRACE(3, i)
        mma_commit(&part_full);
        mma_commit(&mn_empty);
        return true;
      };
      if (ok && nb > 0) ok = issue_scores(0);
      for (int i = 0; i < nb && ok; ++i) {
        // The next block's scores go ahead of this block's gradient MMAs; its
        // buffer was last read by block i - 1's gradient MMAs, issued earlier.
        if (i + 1 < nb) ok = issue_scores(i + 1);
        if (ok) ok = issue_grads(i);
      }
      if (nb > 0) {
        mbar_wait(&kf_empty, (nb - 1) & 1, p.status, kStatusTimeoutEmpty);
        mbar_wait(&mn_empty, (nb - 1) & 1, p.status, kStatusTimeoutEmpty);
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- threads: one key row each
    const int qw = warp % 4;
    const int r = qw * 32 + lane;
    const int ki = k0 + r;
    const int kpos = ki < p.lk ? (p.k_pos ? static_cast<int>(p.k_pos[ki]) : ki) : INT_MAX;
    const uint32_t lb = tmem + (static_cast<uint32_t>(qw * 32) << 16);
    const float* lse_bh = p.lse + (static_cast<long long>(b) * p.heads + h) * p.lq;
    const float* delta_bh = p.delta + (static_cast<long long>(b) * p.heads + h) * p.lq;
    bool ok = true;
    // 3xTF32: add the dV / dK partial (one or two blocks, see the MMA
    // issuer) into the fp32 TMEM masters; the first fold initialises them.
    bool have_master = false;
    auto fold = [&](int i) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const int part = which == 0 ? Cfg::kDVp : Cfg::kDKp;
        const int master = which == 0 ? Cfg::kDVm : Cfg::kDKm;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t a[32], m[32];
          tmem_ld32(lb + part + c * 32, a);
          if (have_master) tmem_ld32(lb + master + c * 32, m);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t)
            m[t] = __float_as_uint((have_master ? __uint_as_float(m[t]) : 0.f) + __uint_as_float(a[t]));
          tmem_st32(lb + master + c * 32, m);
        }
      }
      have_master = true;
      if (threadIdx.x == 64) ABACUS_BWD_TRACE(4, i)
    };
    for (int i = 0; i < nb && ok; ++i) {
      const int entry = block_list[i];
      const int qb = entry & 0xFFFF;
      const bool partial = (entry >> 30) & 1;
      const int buf = (i & 1) * Cfg::kBufCols;
      // This block's lse / Delta / query positions, one query per lane, loaded
      // before the wait for S^T so their latency hides behind it; the row loop
      // below broadcasts them with shuffles.
      float lse_l[NQ / 32], dl_l[NQ / 32];
      int qpos_l[NQ / 32];
#pragma unroll
      for (int c = 0; c < NQ / 32; ++c) {
        const int qi = qb * NQ + c * 32 + lane;
        const int qc = min(qi, p.lq - 1);
        lse_l[c] = __ldg(lse_bh + qc) * kLog2e;
        dl_l[c] = __ldg(delta_bh + qc);
        qpos_l[c] = qi < p.lq ? (p.q_pos ? static_cast<int>(__ldg(p.q_pos + qi)) : qi) : INT_MIN;
      }
      if (!mbar_wait_warp(&st_full[i & 1], (i >> 1) & 1, p.status, kStatusTimeoutAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (threadIdx.x == 64) ABACUS_BWD_TRACE(1, i)
#pragma unroll
      for (int c = 0; c < NQ / 32; ++c) {
        uint32_t sv32[32], dp32[32];
        tmem_ld32(lb + buf + Cfg::kST + c * 32, sv32);
        tmem_ld32(lb + buf + Cfg::kDPT + c * 32, dp32);
        tmem_ld_wait();
        // sv32 / dp32 are overwritten in place with P^T and dS^T (hi parts).
        uint32_t pl[PASSES == 3 ? 32 : 1], dl[PASSES == 3 ? 32 : 1];
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int qpos_t = __shfl_sync(0xffffffffu, qpos_l[c], t);
          const bool valid = !partial || (ki < p.lk && qpos_t >= kpos);
          const float lse2 = __shfl_sync(0xffffffffu, lse_l[c], t);
          const float dl_ = __shfl_sync(0xffffffffu, dl_l[c], t);
          const float pr = valid ? ex2_approx(__uint_as_float(sv32[t]) * p.scale_log2 - lse2) : 0.f;
          const float ds = pr * (__uint_as_float(dp32[t]) - dl_);
          if (PASSES == 3) {
            float a, a_lo, d2, d2_lo;
            split_tf32(pr, a, a_lo);
            split_tf32(ds, d2, d2_lo);
            sv32[t] = __float_as_uint(a);
            pl[t] = __float_as_uint(a_lo);
            dp32[t] = __float_as_uint(d2);
            dl[t] = __float_as_uint(d2_lo);
          } else {
            sv32[t] = __float_as_uint(pr);
            dp32[t] = __float_as_uint(ds);
          }
        }
        tmem_st32(lb + buf + Cfg::kST + c * 32, sv32);
        tmem_st32(lb + buf + Cfg::kDPT + c * 32, dp32);
        if constexpr (PASSES == 3) {
          tmem_st32(lb + buf + Cfg::kST + NQ + c * 32, pl);
          tmem_st32(lb + buf + Cfg::kDPT + NQ + c * 32, dl);
        }
      }
      // Observe the previous block's gradient MMAs (every phase, in order);
      // in 3xTF32 mode fold the partial after every odd block (the next, even
      // block's MMAs start a fresh partial once this thread arrives below).
      if (i > 0) {
        if (!mbar_wait_warp(&part_full, (i - 1) & 1, p.status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        if (PASSES == 3 && ((i - 1) & 1)) {
          tc_fence_after();
          fold(i - 1);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[i & 1]);
      if (threadIdx.x == 64) ABACUS_BWD_TRACE(2, i)
    }
    if (nb > 0 && ok) {
      ok = mbar_wait_warp(&part_full, (nb - 1) & 1, p.status, kStatusTimeoutAccum);
      if (ok && PASSES == 3) {
        tc_fence_after();
        fold(nb - 1);
        tmem_st_wait();
      }
    }
    tc_fence_after();
    // TMEM loads are warp-collective: every lane loads, only valid rows store.
    const bool have = __all_sync(0xffffffffu, ok) && nb > 0;
    {
      float* dvrow;
      float* dkrow;
      if (p.scatter_chunk) {
        const int owner = min(ki, p.lk - 1) / p.scatter_chunk;
        const long long lrow = static_cast<long long>(b) * p.scatter_chunk + (ki - owner * p.scatter_chunk);
        dvrow = p.scatter_dv[owner] + lrow * p.ld_dv + col0;
        dkrow = p.scatter_dk[owner] + lrow * p.ld_dk + col0;
      } else {
        dvrow = p.dv + static_cast<long long>(b * p.lk + ki) * p.ld_dv + col0;
        dkrow = p.dk + static_cast<long long>(b * p.lk + ki) * p.ld_dk + col0;
      }
      const int vcol = PASSES == 3 ? Cfg::kDVm : Cfg::kDVp;
      const int kcol = PASSES == 3 ? Cfg::kDKm : Cfg::kDKp;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t a[32], g[32];
        if (have) {
          tmem_ld32(lb + vcol + c * 32, a);
          tmem_ld32(lb + kcol + c * 32, g);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) a[t] = g[t] = 0u;
        }
        if (ki >= p.lk) continue;
#pragma unroll
        for (int t = 0; t < 32; t += 4) {
          *reinterpret_cast<float4*>(dvrow + c * 32 + t) =
              make_float4(__uint_as_float(a[t]), __uint_as_float(a[t + 1]), __uint_as_float(a[t + 2]), __uint_as_float(a[t + 3]));
          *reinterpret_cast<float4*>(dkrow + c * 32 + t) =
              make_float4(__uint_as_float(g[t]) * p.scale, __uint_as_float(g[t + 1]) * p.scale,
                          __uint_as_float(g[t + 2]) * p.scale, __uint_as_float(g[t + 3]) * p.scale);
        }
      }
    }
    if (p.scatter_chunk) {
      // Publish this 128-key tile to its owner once all four warps stored it.
      __shared__ int tile_ok[4];
      __threadfence_system();
      const bool warp_ok = __all_sync(0xffffffffu, ok);
      if (lane == 0) tile_ok[warp % 4] = warp_ok ? 1 : 0;
      named_barrier_sync(1, 128);
      if (warp == 2 && lane == 0 && tile_ok[0] && tile_ok[1] && tile_ok[2] && tile_ok[3]) {
        red_release_sys_add(p.scatter_counter[k0 / p.scatter_chunk], 1u);
      }
    }
  } else if (PASSES == 3) {
    // ---------------------------------------------------------------- converter
    const int ct = threadIdx.x - 192;
    bool ok = mbar_wait_warp(&kv_full, 0, p.status, kStatusTimeoutFull);
    if (ok) {
      split_tile(sk, sk + Cfg::kKVTile, Cfg::kKVTile, ct, 128);
      split_tile(sv, sv + Cfg::kKVTile, Cfg::kKVTile, ct, 128);
      fence_proxy_async_smem();
      mbar_arrive(&kv_conv);
    }
    // Same order as the producer: K-major block i+1, then MN-major block i.
    for (int step = 0; step <= nb && ok; ++step) {
      if (step < nb) {
        if (!mbar_wait_warp(&kf_full, step & 1, p.status, kStatusTimeoutFull)) break;
        split_tile(tile(0, 0), tile(0, 1), Cfg::kQTile, ct, 128);
        split_tile(tile(2, 0), tile(2, 1), Cfg::kQTile, ct, 128);
        fence_proxy_async_smem();
        mbar_arrive(&kf_conv);
        if (ct == 0) ABACUS_BWD_TRACE(5, step)
      }
      if (step >= 1) {
        if (!mbar_wait_warp(&mn_full, (step - 1) & 1, p.status, kStatusTimeoutFull)) break;
        split_tile(tile(1, 0), tile(1, 1), Cfg::kQTile, ct, 128);
        split_tile(tile(3, 0), tile(3, 1), Cfg::kQTile, ct, 128);
        fence_proxy_async_smem();
        mbar_arrive(&mn_conv);
        if (ct == 0) ABACUS_BWD_TRACE(6, step - 1)
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ============================================================================ dQ
template <int D, int PASSES>
#undef ABACUS_BWD_TRACE

struct DqCfg {
  static constexpr int kOuter = 128;                    // queries per CTA
  static constexpr int kInner = (PASSES == 3 || D == 128) ? 32 : 64;  // keys per block
  static constexpr int kSplit = PASSES == 3 ? 2 : 1;
  static constexpr int kQTile = kOuter * D * 4;         // Q or dO
  static constexpr int kKTile = kInner * D * 4;         // one layout of K or V
  static constexpr int kStageBytes = 3 * kKTile * kSplit;  // K_k, K_mn, V_k [+ lo]
  static constexpr int kSmemRaw = 2 * kQTile * kSplit + kStageBytes + 1024;
  static constexpr int kThreads = PASSES == 3 ? 320 : 192;
  // Register cap for one CTA per SM: each of the 4 SM sub-partitions holds
  // 16384 registers and ceil(warps / 4) of the CTA's warps.
  static constexpr int kWarpsPerSubpartition = (kThreads / 32 + 3) / 4;
  static constexpr int kMaxRegs =
      (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8 > 255 ? 255 : (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8;
  // TMEM: two buffers (blocks alternate) of S and dP (dS hi [, dS lo]), so the
  // next block's score MMAs run while the threads work on this block; then
  // two dQ partial buffers.
  static constexpr int kS = 0, kDP = kInner, kBufCols = kInner + kInner * kSplit;
  static constexpr int kDQ = 2 * kBufCols;
  static constexpr int kCols = kDQ + 2 * D;
  static constexpr uint32_t kTmemCols = kCols <= 256 ? 256 : 512;
  static constexpr int kMaxBlocks = 2048;
  // A CTA that takes all 512 TMEM columns must be alone on its SM (a second
  // one would wait in tcgen05.alloc for the first to finish): ask for more
  // than half of the SM's shared memory.
  static constexpr int kSmemBytes = (kTmemCols == 512 && kSmemRaw < 116 * 1024) ? 116 * 1024 : kSmemRaw;
};

template <int D, int PASSES>
__global__ void __maxnreg__((DqCfg<D, PASSES>::kMaxRegs)) flash_bwd_dq_kernel(const __grid_constant__ BwdParams p) {
  using Cfg = DqCfg<D, PASSES>;
  constexpr int NK = Cfg::kInner;
  static_assert(Cfg::kCols <= 512, "TMEM budget");
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full, q_conv, s_full[2], p_full[2], dq_full[2], dq_empty[2];
  // K_j / V_j tiles in two groups: K-major K and V (S, dP MMAs) and MN-major K
  // (dQ MMA), so the next block's K-major tiles load while this block's dQ runs.
  __shared__ uint64_t kf_full, kf_conv, kf_empty, mn_full, mn_conv, mn_empty;
  __shared__ uint32_t tmem_slot;
  __shared__ int n_blocks;
  __shared__ int abort_flag;
  __shared__ int block_list[Cfg::kMaxBlocks];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) abort_flag = *reinterpret_cast<volatile int*>(p.status);
  __syncthreads();
  if (abort_flag != kStatusOk) return;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sq = smem;                                  // Q hi [, Q lo]
  uint8_t* sdo = smem + Cfg::kQTile * Cfg::kSplit;     // dO hi [, dO lo]
  uint8_t* st = sdo + Cfg::kQTile * Cfg::kSplit;       // K_k, K_mn, V_k, then lo copies
  auto tile = [&](int which, int lo) { return st + (lo * 3 + which) * Cfg::kKTile; };

  const int nmb = (p.lq + 127) / 128;
  const int mb = nmb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int m0 = mb * 128;
  const int q_row0 = b * p.lq + m0;
  const int k_row_base = b * p.lk;
  const int col0 = h * D;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_conv, 128);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 128);
    mbar_init(&p_full[1], 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], 128);
    }
    mbar_init(&kf_full, 1);
    mbar_init(&kf_conv, 128);
    mbar_init(&kf_empty, 1);
    mbar_init(&mn_full, 1);
    mbar_init(&mn_conv, 128);
    mbar_init(&mn_empty, 1);
    fence_mbar_init();
  }
  if (warp == 0) build_block_list<128, NK, Cfg::kMaxBlocks>(p, true, m0, block_list, &n_blocks, lane);
  if (warp == 1) {
    tmem_alloc(&tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int nb = n_blocks;

  if (warp == 0) {
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(&q_full, 2 * Cfg::kQTile);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        tma_load_2d(sq + c * 128 * 128, &p.tma_q_k, &q_full, col0 + 32 * c, q_row0);
        tma_load_2d(sdo + c * 128 * 128, &p.tma_do_k, &q_full, col0 + 32 * c, q_row0);
      }
      // K-major K / V run one block ahead of the MN-major K: block j+1's score
      // MMAs are issued before block j's dQ MMAs.
      int issued_k = 0, issued_mn = 0;
      for (int step = 0; step <= nb; ++step) {
        if (step < nb) {
          const int krow = k_row_base + (block_list[step] & 0xFFFF) * NK;
          if (step >= 1 && !mbar_wait(&kf_empty, (step - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&kf_full, 2 * Cfg::kKTile);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_2d(tile(0, 0) + c * NK * 128, &p.tma_k_k, &kf_full, col0 + 32 * c, krow);
            tma_load_2d(tile(2, 0) + c * NK * 128, &p.tma_v_k, &kf_full, col0 + 32 * c, krow);
          }
          ++issued_k;
        }
        if (step >= 1) {
          const int j = step - 1;
          const int krow = k_row_base + (block_list[j] & 0xFFFF) * NK;
          if (j >= 1 && !mbar_wait(&mn_empty, (j - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&mn_full, Cfg::kKTile);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_2d(tile(1, 0) + c * NK * 128, &p.tma_k_mn, &mn_full, col0 + 32 * c, krow);
          }
          ++issued_mn;
        }
      }
      mbar_wait(&q_full, 0, nullptr, 0);
      if (issued_k > 0) mbar_wait(&kf_full, (issued_k - 1) & 1, nullptr, 0);
      if (issued_mn > 0) mbar_wait(&mn_full, (issued_mn - 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = idesc_tf32(128, NK, false, false);
      constexpr uint32_t idesc_dq = idesc_tf32(128, D, false, true);
      bool ok = mbar_wait(PASSES == 3 ? &q_conv : &q_full, 0, p.status, kStatusTimeoutFull);
      // S = Q K_j^T, dP = dO V_j^T into TMEM buffer j & 1.
      auto issue_scores = [&](int j) -> bool {
        if (!mbar_wait(PASSES == 3 ? &kf_conv : &kf_full, j & 1, p.status, kStatusTimeoutFull)) return false;
        tc_fence_after();
        const int sb = (j & 1) * Cfg::kBufCols;
#pragma unroll
        for (int pair = 0; pair < 2; ++pair) {
          const uint32_t a_hi = smem_u32(pair == 0 ? sq : sdo);
          const uint32_t b_hi = smem_u32(tile(pair == 0 ? 0 : 2, 0));
          const uint32_t b_lo = smem_u32(tile(pair == 0 ? 0 : 2, 1));
          const uint32_t d = tmem + sb + (pair == 0 ? Cfg::kS : Cfg::kDP);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint32_t ao = c * 128 * 128 + ks * 32;
              const uint32_t bo = c * NK * 128 + ks * 32;
              const uint32_t acc = (c | ks) ? 1u : 0u;
              if (PASSES == 3) {
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + Cfg::kQTile + ao), desc_kmajor_sw128(b_hi + bo), idesc_s, acc);
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + ao), desc_kmajor_sw128(b_lo + bo), idesc_s, 1u);
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + ao), desc_kmajor_sw128(b_hi + bo), idesc_s, 1u);
              } else {
                mma_tf32_ss(d, desc_kmajor_sw128(a_hi + ao), desc_kmajor_sw128(b_hi + bo), idesc_s, acc);
              }
            }
          }
        }
        mma_commit(&s_full[j & 1]);
        mma_commit(&kf_empty);
        return true;
      };
      // dQ_j = dS_j K_j into partial buffer j & 1, A from TMEM buffer j & 1.
      auto issue_dq = [&](int j) -> bool {
        const int buf = j & 1;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.status, kStatusTimeoutAccum)) return false;
        if (!mbar_wait(PASSES == 3 ? &mn_conv : &mn_full, j & 1, p.status, kStatusTimeoutFull)) return false;
        if (j >= 2 && !mbar_wait(&dq_empty[buf], ((j >> 1) - 1) & 1, p.status, kStatusTimeoutAccum)) return false;
        tc_fence_after();
        const uint32_t a = tmem + buf * Cfg::kBufCols + Cfg::kDP;
        const uint32_t bh = smem_u32(tile(1, 0));
        const uint32_t bl = smem_u32(tile(1, 1));
        const uint32_t d = tmem + Cfg::kDQ + buf * D;
#pragma unroll
        for (int ks = 0; ks < NK / 8; ++ks) {
          const uint64_t kbd = desc_mnmajor_sw128_32b(bh + ks * 1024, NK * 128);
          const uint32_t acc = ks ? 1u : 0u;
          if (PASSES == 3) {
            const uint64_t kl = desc_mnmajor_sw128_32b(bl + ks * 1024, NK * 128);
            mma_tf32_ts(d, a + NK + ks * 8, kbd, idesc_dq, acc);
            mma_tf32_ts(d, a + ks * 8, kl, idesc_dq, 1u);
            mma_tf32_ts(d, a + ks * 8, kbd, idesc_dq, 1u);
          } else {
            mma_tf32_ts(d, a + ks * 8, kbd, idesc_dq, acc);
          }
        }
        mma_commit(&dq_full[buf]);
        mma_commit(&mn_empty);
        return true;
      };
      if (ok && nb > 0) ok = issue_scores(0);
      for (int j = 0; j < nb && ok; ++j) {
        // The next block's scores go ahead of this block's dQ MMAs; their
        // buffer was last read by block j - 1's dQ MMAs, issued earlier.
        if (j + 1 < nb) ok = issue_scores(j + 1);
        if (ok) ok = issue_dq(j);
      }
      if (nb > 0) {
        mbar_wait(&kf_empty, (nb - 1) & 1, p.status, kStatusTimeoutEmpty);
        mbar_wait(&mn_empty, (nb - 1) & 1, p.status, kStatusTimeoutEmpty);
      }
    }
  } else if (warp < 6) {
    const int qw = warp % 4;
    const int r = qw * 32 + lane;
    const int qi = m0 + r;
    const int qc = min(qi, p.lq - 1);
    const int qpos = qi < p.lq ? (p.q_pos ? static_cast<int>(p.q_pos[qi]) : qi) : INT_MIN;
    const uint32_t lb = tmem + (static_cast<uint32_t>(qw * 32) << 16);
    const long long bh = static_cast<long long>(b) * p.heads + h;
    const float lse2 = p.lse[bh * p.lq + qc] * kLog2e;
    const float dl_ = p.delta[bh * p.lq + qc];
    float dq[D];
#pragma unroll
    for (int t = 0; t < D; ++t) dq[t] = 0.f;
    bool ok = true;
    auto fold = [&](int j) -> bool {
      const int buf = j & 1;
      if (!mbar_wait_warp(&dq_full[buf], (j >> 1) & 1, p.status, kStatusTimeoutAccum)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(lb + Cfg::kDQ + buf * D + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) dq[c * 32 + t] += __uint_as_float(v[t]);
      }
      tc_fence_before();
      mbar_arrive(&dq_empty[buf]);
      return true;
    };
    for (int j = 0; j < nb && ok; ++j) {
      const int entry = block_list[j];
      const int kbk = entry & 0xFFFF;
      const bool partial = (entry >> 30) & 1;
      const int sb = (j & 1) * Cfg::kBufCols;
      if (!mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1, p.status, kStatusTimeoutAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < NK / 32; ++c) {
        uint32_t sv32[32], dp32[32];
        tmem_ld32(lb + sb + Cfg::kS + c * 32, sv32);
        tmem_ld32(lb + sb + Cfg::kDP + c * 32, dp32);
        tmem_ld_wait();
        // dp32 is overwritten in place with dS (hi part); sv32 with dS lo.
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int ki = kbk * NK + c * 32 + t;
          bool valid = true;
          if (partial) valid = qi < p.lq && ki < p.lk && (p.k_pos ? static_cast<int>(__ldg(p.k_pos + ki)) : ki) <= qpos;
          const float pr = valid ? ex2_approx(__uint_as_float(sv32[t]) * p.scale_log2 - lse2) : 0.f;
          const float ds = pr * (__uint_as_float(dp32[t]) - dl_);
          if (PASSES == 3) {
            float a, a_lo;
            split_tf32(ds, a, a_lo);
            dp32[t] = __float_as_uint(a);
            sv32[t] = __float_as_uint(a_lo);
          } else {
            dp32[t] = __float_as_uint(ds);
          }
        }
        tmem_st32(lb + sb + Cfg::kDP + c * 32, dp32);
        if (PASSES == 3) tmem_st32(lb + sb + Cfg::kDP + NK + c * 32, sv32);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      if (j >= 1 && !fold(j - 1)) ok = false;
    }
    if (ok && nb > 0) ok = fold(nb - 1);
    if (qi < p.lq) {
      float* row = p.dq + static_cast<long long>(q_row0 + r) * p.ld_dq + col0;
#pragma unroll
      for (int t = 0; t < D; t += 4)
        *reinterpret_cast<float4*>(row + t) =
            make_float4(dq[t] * p.scale, dq[t + 1] * p.scale, dq[t + 2] * p.scale, dq[t + 3] * p.scale);
    }
  } else if (PASSES == 3) {
    const int ct = threadIdx.x - 192;
    bool ok = mbar_wait_warp(&q_full, 0, p.status, kStatusTimeoutFull);
    if (ok) {
      split_tile(sq, sq + Cfg::kQTile, Cfg::kQTile, ct, 128);
      split_tile(sdo, sdo + Cfg::kQTile, Cfg::kQTile, ct, 128);
      fence_proxy_async_smem();
      mbar_arrive(&q_conv);
    }
    // Same order as the producer: K-major block j+1, then MN-major block j.
    for (int step = 0; step <= nb && ok; ++step) {
      if (step < nb) {
        if (!mbar_wait_warp(&kf_full, step & 1, p.status, kStatusTimeoutFull)) break;
        split_tile(tile(0, 0), tile(0, 1), Cfg::kKTile, ct, 128);
        split_tile(tile(2, 0), tile(2, 1), Cfg::kKTile, ct, 128);
        fence_proxy_async_smem();
        mbar_arrive(&kf_conv);
      }
      if (step >= 1) {
        if (!mbar_wait_warp(&mn_full, (step - 1) & 1, p.status, kStatusTimeoutFull)) break;
        split_tile(tile(1, 0), tile(1, 1), Cfg::kKTile, ct, 128);
        fence_proxy_async_smem();
        mbar_arrive(&mn_conv);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace attn
}  // namespace abacus
