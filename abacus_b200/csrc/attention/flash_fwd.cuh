// Causal flash-attention forward on tcgen05 (kind::tf32), fp32 in / out.
//
// One CTA = 128 queries of one (batch, head). Keys are visited in blocks of
// 64; blocks entirely in the masked future are skipped (positions may be the
// global zigzag positions of context parallelism).
//
//   warp 0      TMA producer: Q once, then K_j and V_j into two 2-slot rings
//               with their own barriers: a K slot is free as soon as S_j has
//               read it, a V slot once PV_j has, so K runs one block ahead
//   warp 1      TMEM allocator + single-thread MMA issuer
//                 S_j  = Q K_j^T          (A, B from smem, K-major)
//                 PV_j = P_j V_j          (A = P from TMEM, B = V MN-major)
//   warps 2-5   softmax: one query row per thread. Reads S_j from TMEM,
//               masks / scales, online max & sum, writes P_j into TMEM (the
//               columns S_j came from), then folds PV_{j-1} into its fp32
//               register accumulator with the online-softmax rescale.
//   warps 6-9   (3xTF32 only) split converter: each landed Q / K / V tile is
//               rewritten as hi (in place) and lo, so every product is
//               lo*hi + hi*lo + hi*hi.
//
// P_j never touches shared or global memory, the (L, L) score matrix is never
// materialised, and each PV_j lands in a fresh TMEM buffer that is added to
// the register accumulator with round-to-nearest fp32 adds (the tensor core's
// own accumulation spans one 64-key block only).
//
// TMEM columns: SP[2] (S, then P hi [+ P lo]) and PV[2].
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cfloat>
#include <cstdint>
#include "../common/sm100.cuh"

namespace abacus {
namespace attn {

constexpr int kBlockM = 128;  // queries per CTA (one per softmax thread)
constexpr int kBlockN = 64;   // keys per block

struct FwdParams {
  CUtensorMap tma_q;   // box {32, 128} over (B*Lq, ld_q), SWIZZLE_128B
  CUtensorMap tma_k;   // box {32, 64}  over (B*Lk, ld_k), SWIZZLE_128B
  CUtensorMap tma_v;   // box {32, 64}  over (B*Lk, ld_v), SWIZZLE_128B_ATOM_32B
  float* out;          // (B*Lq, ld_o)
  long long ld_o;
  float* lse;          // (B, H, Lq)
  const int64_t* q_pos;  // (Lq,) or null (then position = index)
  const int64_t* k_pos;  // (Lk,) or null
  int batch, heads, lq, lk;
  float scale_log2;    // softmax scale * log2(e)
  // Context parallel: K / V rows are pushed here by their owning ranks; a CTA
  // starts once every other rank published `wait_epoch` (null: no wait).
  const int* wait_flags;
  int wait_epoch, wait_world, wait_self;
  int* status;
  // Optional phase trace (clock64 stamps of CTA (0, 0, 0), slot * 64 + block):
  // 0 K/V load issued, 1 K/V split, 2 S issued, 3 PV issued, 4 S seen by the
  // softmax, 5 P written, 6 PV seen, 7 PV folded, 8 (+0 start, +1 set-up, +2 end).
  long long* trace;
};

template <int D, int PASSES>
struct FwdCfg {
  static constexpr int kQBytes = kBlockM * D * 4;
  static constexpr int kKBytes = kBlockN * D * 4;
  static constexpr int kVBytes = kBlockN * D * 4;
  static constexpr int kSplit = PASSES == 3 ? 2 : 1;
  static constexpr int kStages = 2;
  static constexpr int kStageBytes = (kKBytes + kVBytes) * kSplit;
  static constexpr int kSmemRaw = kQBytes * kSplit + kStages * kStageBytes + 1024;
  // 3xTF32 at head_dim 64: each query row's softmax is shared by two warps
  // (two warpgroups, 32 of the 64 key columns and 32 of the 64 output columns
  // each), so a key block's exp / split / TMEM work is halved per thread; the
  // row maxima and, at the end, the row sums are exchanged in shared memory.
  // Warpgroups: 0 producer + MMA, 1 and 2 softmax halves, 3 converter, with a
  // setmaxnreg split of 128 x (72 + 168 + 168 + 104) = 65536 registers.
  static constexpr int kHalves = (PASSES == 3 && D == 64) ? 2 : 1;
  static constexpr int kCtrlWarps = kHalves == 2 ? 4 : 2;
  static constexpr int kSoftWarp0 = kCtrlWarps;
  static constexpr int kConvWarp0 = kSoftWarp0 + 4 * kHalves;
  static constexpr uint32_t kRegsCtrl = 72, kRegsSoft = 168, kRegsConv = 104;
  static constexpr int kThreads = kHalves == 2 ? 512 : (PASSES == 3 ? 320 : 192);
  static_assert(kHalves == 1 || 128 * (kRegsCtrl + 2 * kRegsSoft + kRegsConv) == kThreads * 128,
                "warpgroup register budgets must add up to the launch's 65536");
  // Register cap for one CTA per SM: each of the 4 SM sub-partitions holds
  // 16384 registers and ceil(warps / 4) of the CTA's warps.
  static constexpr int kWarpsPerSubpartition = (kThreads / 32 + 3) / 4;
  static constexpr int kMaxRegs =
      (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8 > 255 ? 255 : (16384 / (32 * kWarpsPerSubpartition)) / 8 * 8;
  static constexpr int kSPCols = kBlockN * (PASSES == 3 ? 2 : 1);  // S / P hi [/ P lo]
  static constexpr int kPVBase = 2 * kSPCols;
  static constexpr int kCols = kPVBase + 2 * D;
  static constexpr uint32_t kTmemCols = kCols <= 256 ? 256 : 512;
  static constexpr int kMaxBlocks = 2048;  // key blocks per sequence (Lk <= 131072)
  // A CTA that takes all 512 TMEM columns must be alone on its SM (a second
  // one would wait in tcgen05.alloc for the first to finish): ask for more
  // than half of the SM's shared memory.
  static constexpr int kSmemBytes = (kTmemCols == 512 && kSmemRaw < 116 * 1024) ? 116 * 1024 : kSmemRaw;
};


template <int D, int PASSES>
__global__ void __maxnreg__((FwdCfg<D, PASSES>::kMaxRegs)) flash_fwd_kernel(const __grid_constant__ FwdParams p) {
  using Cfg = FwdCfg<D, PASSES>;
  static_assert(D % 32 == 0 && D <= 128, "head_dim must be 32, 64, 96 or 128");
  static_assert(Cfg::kCols <= 512, "TMEM budget");
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full, q_conv;
  __shared__ uint64_t k_full[2], k_conv[2], k_empty[2], v_full[2], v_conv[2], v_empty[2];
  __shared__ uint64_t s_full[2], p_full[2], pv_full[2], pv_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int n_blocks;
  __shared__ int block_list[Cfg::kMaxBlocks];  // key block index | (needs_mask << 30)

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool traced = p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;

#define ABACUS_FWD_TRACE(slot, j) \
  if (traced && (j) < 64) p.trace[(slot) * 64 + (j)] = clock64();
  if (threadIdx.x == 0) ABACUS_FWD_TRACE(8, 0)
  // Abort early (uniformly for the whole CTA) if an earlier kernel on this
  // device already recorded an error.
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = *reinterpret_cast<volatile int*>(p.status);
    if (abort_flag == kStatusOk && p.wait_flags != nullptr) {
      for (int r = 0; r < p.wait_world; ++r) {
        if (r != p.wait_self && !wait_flag_geq(p.wait_flags + r, p.wait_epoch, p.status)) {
          abort_flag = kStatusTimeoutPeer;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (abort_flag != kStatusOk) return;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sq = smem;                                   // Q hi [| Q lo]
  uint8_t* skv = smem + Cfg::kQBytes * Cfg::kSplit;     // stages: K hi, V hi [, K lo, V lo]
  auto k_hi = [&](int s) { return skv + s * Cfg::kStageBytes; };
  auto v_hi = [&](int s) { return skv + s * Cfg::kStageBytes + Cfg::kKBytes; };
  auto k_lo = [&](int s) { return skv + s * Cfg::kStageBytes + Cfg::kKBytes + Cfg::kVBytes; };
  auto v_lo = [&](int s) { return skv + s * Cfg::kStageBytes + 2 * Cfg::kKBytes + Cfg::kVBytes; };

  // Heavy (late) query blocks first: causal work grows with the block index.
  const int num_mb = (p.lq + kBlockM - 1) / kBlockM;
  const int mb = num_mb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int m0 = mb * kBlockM;
  const int q_row0 = b * p.lq + m0;  // row in the (B*Lq) matrix
  const int k_row0 = b * p.lk;
  const int col0 = h * D;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_conv, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_conv[i], 128);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_conv[i], 128);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128 * Cfg::kHalves);
      mbar_init(&pv_full[i], 1);
      mbar_init(&pv_empty[i], 128 * Cfg::kHalves);
    }
    fence_mbar_init();
  }
  // Key blocks this query block must visit, with a flag for blocks that
  // straddle the causal boundary (need per-element masking).
  if (warp == 0) {
    // Query position range of this block.
    int qmin = INT_MAX, qmax = INT_MIN;
    for (int i = lane; i < kBlockM; i += 32) {
      const int qi = m0 + i;
      if (qi < p.lq) {
        const int pos = p.q_pos ? static_cast<int>(p.q_pos[qi]) : qi;
        qmin = min(qmin, pos);
        qmax = max(qmax, pos);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      qmin = min(qmin, __shfl_xor_sync(0xffffffffu, qmin, o));
      qmax = max(qmax, __shfl_xor_sync(0xffffffffu, qmax, o));
    }
    const int nkb = (p.lk + kBlockN - 1) / kBlockN;
    int count = 0;
    for (int base = 0; base < nkb; base += 32) {
      const int kb = base + lane;
      bool keep = false, partial = false;
      if (kb < nkb) {
        int kmin = INT_MAX, kmax = INT_MIN;
        for (int i = 0; i < kBlockN; ++i) {
          const int ki = kb * kBlockN + i;
          if (ki < p.lk) {
            const int pos = p.k_pos ? static_cast<int>(p.k_pos[ki]) : ki;
            kmin = min(kmin, pos);
            kmax = max(kmax, pos);
          }
        }
        keep = kmin <= qmax;
        partial = kmax > qmin || (kb * kBlockN + kBlockN > p.lk);
      }
      const unsigned keep_mask = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const int slot = count + __popc(keep_mask & ((1u << lane) - 1u));
        if (slot < Cfg::kMaxBlocks) block_list[slot] = kb | (partial ? (1 << 30) : 0);
      }
      count += __popc(keep_mask);
    }
    if (lane == 0) n_blocks = min(count, Cfg::kMaxBlocks);
    if (lane == 0 && count > Cfg::kMaxBlocks) atomicCAS(p.status, kStatusOk, kStatusBadArgs);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int nb = n_blocks;
  if (threadIdx.x == 0) ABACUS_FWD_TRACE(8, 1)

  if (warp < Cfg::kCtrlWarps) {
  if constexpr (Cfg::kHalves == 2) regs_decrease<Cfg::kRegsCtrl>();
  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one_sync()) {
      tma_prefetch_desc(&p.tma_q);
      tma_prefetch_desc(&p.tma_k);
      tma_prefetch_desc(&p.tma_v);
      mbar_arrive_expect_tx(&q_full, Cfg::kQBytes);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tma_load_2d(sq + c * kBlockM * 128, &p.tma_q, &q_full, col0 + 32 * c, q_row0);
      // K runs one block ahead of V: K_j is needed by S_j, V_j only by PV_j,
      // which follows the softmax of block j.
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          const int s = j & 1;
          if (j >= 2 && !mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
          ABACUS_FWD_TRACE(0, j)
          const int krow = k_row0 + (block_list[j] & 0xFFFF) * kBlockN;
          mbar_arrive_expect_tx(&k_full[s], Cfg::kKBytes);
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            tma_load_2d(k_hi(s) + c * kBlockN * 128, &p.tma_k, &k_full[s], col0 + 32 * c, krow);
          ++issued_k;
        }
        if (j >= 1) {
          const int jv = j - 1, s = jv & 1;
          if (jv >= 2 && !mbar_wait(&v_empty[s], ((jv >> 1) - 1) & 1, p.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int vrow = k_row0 + (block_list[jv] & 0xFFFF) * kBlockN;
          mbar_arrive_expect_tx(&v_full[s], Cfg::kVBytes);
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            tma_load_2d(v_hi(s) + c * kBlockN * 128, &p.tma_v, &v_full[s], col0 + 32 * c, vrow);
          ++issued_v;
        }
      }
      // No TMA may still be writing this CTA's shared memory at exit.
      mbar_wait(&q_full, 0, nullptr, 0);
      for (int j = max(0, issued_k - 2); j < issued_k; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, 0);
      for (int j = max(0, issued_v - 2); j < issued_v; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = idesc_tf32(kBlockM, kBlockN, false, false);
      constexpr uint32_t idesc_pv = idesc_tf32(kBlockM, D, false, true);
      bool ok = mbar_wait(PASSES == 3 ? &q_conv : &q_full, 0, p.status, kStatusTimeoutFull);
      // S_j = Q K_j^T into SP[j & 1].
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(PASSES == 3 ? &k_conv[s] : &k_full[s], (j >> 1) & 1, p.status, kStatusTimeoutFull))
          return false;
        ABACUS_FWD_TRACE(2, j)
        tc_fence_after();
        const uint32_t d = tmem + s * Cfg::kSPCols;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t qa = smem_u32(sq) + c * kBlockM * 128 + ks * 32;
            const uint32_t kb = smem_u32(k_hi(s)) + c * kBlockN * 128 + ks * 32;
            const uint32_t acc = (c | ks) ? 1u : 0u;
            if (PASSES == 3) {
              const uint32_t ql = qa + Cfg::kQBytes;
              const uint32_t kl = kb + (Cfg::kKBytes + Cfg::kVBytes);
              mma_tf32_ss(d, desc_kmajor_sw128(ql), desc_kmajor_sw128(kb), idesc_s, acc);
              mma_tf32_ss(d, desc_kmajor_sw128(qa), desc_kmajor_sw128(kl), idesc_s, 1u);
              mma_tf32_ss(d, desc_kmajor_sw128(qa), desc_kmajor_sw128(kb), idesc_s, 1u);
            } else {
              mma_tf32_ss(d, desc_kmajor_sw128(qa), desc_kmajor_sw128(kb), idesc_s, acc);
            }
          }
        }
        mma_commit(&s_full[s]);
        mma_commit(&k_empty[s]);
        return true;
      };
      // PV_j = P_j V_j into PV[j & 1].
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&p_full[s], (j >> 1) & 1, p.status, kStatusTimeoutAccum)) return false;
        if (j >= 2 && !mbar_wait(&pv_empty[s], ((j >> 1) - 1) & 1, p.status, kStatusTimeoutAccum)) return false;
        if (!mbar_wait(PASSES == 3 ? &v_conv[s] : &v_full[s], (j >> 1) & 1, p.status, kStatusTimeoutFull)) return false;
        ABACUS_FWD_TRACE(3, j)
        tc_fence_after();
        const uint32_t d = tmem + Cfg::kPVBase + s * D;
        const uint32_t p_hi = tmem + s * Cfg::kSPCols;
        const uint32_t v_base = smem_u32(v_hi(s));
#pragma unroll
        for (int ks = 0; ks < kBlockN / 8; ++ks) {
          const uint64_t vb = desc_mnmajor_sw128_32b(v_base + ks * 1024, kBlockN * 128);
          const uint32_t acc = ks ? 1u : 0u;
          if (PASSES == 3) {
            const uint64_t vl = desc_mnmajor_sw128_32b(v_base + Cfg::kKBytes + Cfg::kVBytes + ks * 1024, kBlockN * 128);
            mma_tf32_ts(d, p_hi + kBlockN + ks * 8, vb, idesc_pv, acc);  // P lo * V hi
            mma_tf32_ts(d, p_hi + ks * 8, vl, idesc_pv, 1u);             // P hi * V lo
            mma_tf32_ts(d, p_hi + ks * 8, vb, idesc_pv, 1u);             // P hi * V hi
          } else {
            mma_tf32_ts(d, p_hi + ks * 8, vb, idesc_pv, acc);
          }
        }
        mma_commit(&pv_full[s]);
        mma_commit(&v_empty[s]);
        return true;
      };
      for (int j = 0; j < nb && ok; ++j) {
        ok = issue_s(j);
        if (ok && j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && nb >= 1) ok = issue_pv(nb - 1);
      // Drain: every commit lands before this CTA releases its shared memory.
      if (nb >= 1) {
        for (int j = max(0, nb - 2); j < nb; ++j) {
          mbar_wait(&k_empty[j & 1], (j >> 1) & 1, p.status, kStatusTimeoutEmpty);
          mbar_wait(&v_empty[j & 1], (j >> 1) & 1, p.status, kStatusTimeoutEmpty);
        }
      }
    }
  }  // warps 2 and 3 of warpgroup 0 (split softmax) have no role
  } else if (Cfg::kHalves == 2 && warp < Cfg::kConvWarp0) {
    // ------------------------------------------------------- softmax, split
    // Warp w of warpgroup 1 and warp w of warpgroup 2 hold the same 32 query
    // rows (TMEM lanes); half h takes S / P columns [32 h, 32 h + 32) of each
    // key block and output columns [32 h, 32 h + 32).
    regs_increase<Cfg::kRegsSoft>();
    __shared__ float xmax[2][2][kBlockM];  // [block parity][half][row]
    __shared__ float xsum[2][kBlockM];
    const int q = warp % 4;
    const int half = (warp - Cfg::kSoftWarp0) / 4;
    const int r = q * 32 + lane;
    const int qi = m0 + r;
    const int qpos = qi < p.lq ? (p.q_pos ? static_cast<int>(p.q_pos[qi]) : qi) : INT_MIN;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const bool tracer = threadIdx.x == Cfg::kSoftWarp0 * 32;
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0.f;
    float m = -FLT_MAX, l = 0.f, alpha_prev = 0.f;
    // After a failed wait the warp keeps meeting its partner at every row
    // exchange (a named barrier has no time limit) but skips the work.
    bool dead = false;
    for (int j = 0; j <= nb; ++j) {
      float alpha = 1.f;
      if (j < nb) {
        const int s = j & 1;
        const int entry = block_list[j];
        const int kb = entry & 0xFFFF;
        const bool partial = (entry >> 30) & 1;
        if (!dead && !mbar_wait_warp(&s_full[s], (j >> 1) & 1, p.status, kStatusTimeoutAccum)) dead = true;
        if (tracer) ABACUS_FWD_TRACE(4, j)
        tc_fence_after();
        float sv[32];
        float bmax = -FLT_MAX;
        if (!dead) {
          uint32_t v[32];
          tmem_ld32(lane_base + s * Cfg::kSPCols + half * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(v[i]) * p.scale_log2;
          if (partial) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int ki = kb * kBlockN + half * 32 + i;
              const bool valid = ki < p.lk && (p.k_pos ? static_cast<int>(__ldg(p.k_pos + ki)) : ki) <= qpos;
              if (!valid) sv[i] = -FLT_MAX;
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) bmax = fmaxf(bmax, sv[i]);
        }
        xmax[j & 1][half][r] = bmax;
        named_barrier_sync(1 + q, 64);
        bmax = fmaxf(bmax, xmax[j & 1][half ^ 1][r]);
        const float m_new = fmaxf(m, bmax);
        alpha = (m == -FLT_MAX) ? 0.f : ex2_approx(m - m_new);
        if (!dead) {
          float bsum = 0.f;
          uint32_t vh[32], vl[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float e = (sv[i] == -FLT_MAX) ? 0.f : ex2_approx(sv[i] - m_new);
            bsum += e;
            float hi, lo;
            split_tf32(e, hi, lo);
            vh[i] = __float_as_uint(hi);
            vl[i] = __float_as_uint(lo);
          }
          tmem_st32(lane_base + s * Cfg::kSPCols + half * 32, vh);
          tmem_st32(lane_base + s * Cfg::kSPCols + kBlockN + half * 32, vl);
          l = l * alpha + bsum;
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(&p_full[s]);
        }
        m = m_new;
        if (tracer) ABACUS_FWD_TRACE(5, j)
      }
      if (j >= 1 && !dead) {
        // Fold this half of PV_{j-1}: o = o * alpha_{j-1} + PV_{j-1}.
        const int s = (j - 1) & 1;
        if (!mbar_wait_warp(&pv_full[s], ((j - 1) >> 1) & 1, p.status, kStatusTimeoutAccum)) {
          dead = true;
        } else {
          if (tracer) ABACUS_FWD_TRACE(6, j - 1)
          tc_fence_after();
          uint32_t v[32];
          tmem_ld32(lane_base + Cfg::kPVBase + s * D + half * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = o[i] * alpha_prev + __uint_as_float(v[i]);
          tc_fence_before();
          mbar_arrive(&pv_empty[s]);
          if (tracer) ABACUS_FWD_TRACE(7, j - 1)
        }
      }
      alpha_prev = alpha;
    }
    // The row sum is the two halves' sums.
    xsum[half][r] = l;
    named_barrier_sync(1 + q, 64);
    l += xsum[half ^ 1][r];
    if (!dead && qi < p.lq) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float* orow = p.out + static_cast<long long>(q_row0 + r) * p.ld_o + col0 + half * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(orow + i) = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      if (half == 0) p.lse[(static_cast<long long>(b) * p.heads + h) * p.lq + qi] = (m + log2f(l)) * 0.69314718055994531f;
    }
  } else if (warp < Cfg::kConvWarp0) {
    // ---------------------------------------------------------------- softmax
    const int q = warp % 4;
    const int r = q * 32 + lane;  // row within the block == TMEM lane
    const int qi = m0 + r;
    const int qpos = qi < p.lq ? (p.q_pos ? static_cast<int>(p.q_pos[qi]) : qi) : INT_MIN;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    float m = -FLT_MAX, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    for (int j = 0; j <= nb && ok; ++j) {
      float alpha = 1.f;
      if (j < nb) {
        const int s = j & 1;
        const int entry = block_list[j];
        const int kb = entry & 0xFFFF;
        const bool partial = (entry >> 30) & 1;
        if (!mbar_wait_warp(&s_full[s], (j >> 1) & 1, p.status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 64) ABACUS_FWD_TRACE(4, j)
        tc_fence_after();
        // Scaled, masked scores of 32 columns of S_j (re-read from TMEM, which
        // is cheaper than keeping 64 scores live in registers).
        auto load_scores = [&](int c, float (&sv)[32]) {
          uint32_t v[32];
          tmem_ld32(lane_base + s * Cfg::kSPCols + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(v[i]) * p.scale_log2;
          if (partial) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int ki = kb * kBlockN + c * 32 + i;
              const bool valid = ki < p.lk && (p.k_pos ? static_cast<int>(__ldg(p.k_pos + ki)) : ki) <= qpos;
              if (!valid) sv[i] = -FLT_MAX;
            }
          }
        };
        float bmax = -FLT_MAX;
#pragma unroll
        for (int c = 0; c < kBlockN / 32; ++c) {
          float sv[32];
          load_scores(c, sv);
#pragma unroll
          for (int i = 0; i < 32; ++i) bmax = fmaxf(bmax, sv[i]);
        }
        const float m_new = fmaxf(m, bmax);
        alpha = (m == -FLT_MAX) ? 0.f : ex2_approx(m - m_new);
        float bsum = 0.f;
        // P into the TMEM columns S came from (and the next kBlockN for P lo).
#pragma unroll
        for (int c = 0; c < kBlockN / 32; ++c) {
          float sv[32];
          load_scores(c, sv);
          uint32_t vh[32];
          uint32_t vl[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float e = (sv[i] == -FLT_MAX) ? 0.f : ex2_approx(sv[i] - m_new);
            bsum += e;
            if (PASSES == 3) {
              float hi, lo;
              split_tf32(e, hi, lo);
              vh[i] = __float_as_uint(hi);
              vl[i] = __float_as_uint(lo);
            } else {
              vh[i] = __float_as_uint(e);
            }
          }
          tmem_st32(lane_base + s * Cfg::kSPCols + c * 32, vh);
          if (PASSES == 3) tmem_st32(lane_base + s * Cfg::kSPCols + kBlockN + c * 32, vl);
        }
        l = l * alpha + bsum;
        m = m_new;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[s]);
        if (threadIdx.x == 64) ABACUS_FWD_TRACE(5, j)
      }
      if (j >= 1) {
        // Fold PV_{j-1}: o = o * alpha_{j-1} + PV_{j-1}.
        const int s = (j - 1) & 1;
        if (!mbar_wait_warp(&pv_full[s], ((j - 1) >> 1) & 1, p.status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 64) ABACUS_FWD_TRACE(6, j - 1)
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(lane_base + Cfg::kPVBase + s * D + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha_prev + __uint_as_float(v[i]);
        }
        tc_fence_before();
        mbar_arrive(&pv_empty[s]);
        if (threadIdx.x == 64) ABACUS_FWD_TRACE(7, j - 1)
      }
      alpha_prev = alpha;
    }
    if (ok && qi < p.lq) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float* orow = p.out + static_cast<long long>(q_row0 + r) * p.ld_o + col0;
#pragma unroll
      for (int i = 0; i < D; i += 4)
        *reinterpret_cast<float4*>(orow + i) = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      // Natural-log LSE of the scaled scores.
      p.lse[(static_cast<long long>(b) * p.heads + h) * p.lq + qi] = (m + log2f(l)) * 0.69314718055994531f;
    }
  } else if (PASSES == 3) {
    // ---------------------------------------------------------------- converter
    if constexpr (Cfg::kHalves == 2) regs_decrease<Cfg::kRegsConv>();
    const int ct = threadIdx.x - Cfg::kConvWarp0 * 32;
    auto split = [&](uint8_t* hi_buf, uint8_t* lo_buf, int bytes) {
      float4* hi = reinterpret_cast<float4*>(hi_buf);
      float4* lo = reinterpret_cast<float4*>(lo_buf);
      for (int i = ct; i < bytes / 16; i += 128) {
        // hi stays raw (the MMA truncates it to tf32); only lo is written.
        const float4 x = hi[i];
        lo[i] = make_float4(tf32_lo_of_raw(x.x), tf32_lo_of_raw(x.y), tf32_lo_of_raw(x.z), tf32_lo_of_raw(x.w));
      }
    };
    bool ok = mbar_wait_warp(&q_full, 0, p.status, kStatusTimeoutFull);
    if (ok) {
      split(sq, sq + Cfg::kQBytes, Cfg::kQBytes);
      fence_proxy_async_smem();
      mbar_arrive(&q_conv);
    }
    // Same order as the producer: K_j, then V_{j-1}.
    for (int j = 0; j <= nb && ok; ++j) {
      if (j < nb) {
        const int s = j & 1;
        if (!mbar_wait_warp(&k_full[s], (j >> 1) & 1, p.status, kStatusTimeoutFull)) break;
        split(k_hi(s), k_lo(s), Cfg::kKBytes);
        fence_proxy_async_smem();
        mbar_arrive(&k_conv[s]);
        if (ct == 0) ABACUS_FWD_TRACE(1, j)
      }
      if (j >= 1) {
        const int s = (j - 1) & 1;
        if (!mbar_wait_warp(&v_full[s], ((j - 1) >> 1) & 1, p.status, kStatusTimeoutFull)) break;
        split(v_hi(s), v_lo(s), Cfg::kVBytes);
        fence_proxy_async_smem();
        mbar_arrive(&v_conv[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) ABACUS_FWD_TRACE(8, 2)
#undef ABACUS_FWD_TRACE
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace attn
}  // namespace abacus
