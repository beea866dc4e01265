// tcgen05 (kind::tf32) GEMM for sm_100a: C[M,N] = A[M,K] * B[K,N] in fp32
// storage with an fp32 TMEM accumulator.
//
// * One CTA computes one 128 x BN output tile.
// * Warp 0: TMA producer. Warp 1: TMEM allocator + single-thread MMA issuer.
//   Epilogue warpgroup (warps 2-5; 4-7 in 3xTF32 mode): TMEM -> registers ->
//   global. Warps 8-15 (3xTF32 only, two warpgroups taking alternate
//   k-tiles): split-precision converter: A rows go to TMEM as hi = tf32(x) and
//   lo = tf32(x - hi); B stays raw in shared memory (the MMA reads it as its
//   truncated tf32 hi part) and lo = tf32(x - trunc(x)) is written beside it,
//   so the MMA warp can issue lo*hi + hi*lo + hi*hi (fp32-level accuracy).
// * Operands may be K-major (row-major along K; TMA SWIZZLE_128B) or MN-major
//   (row-major along M/N; TMA SWIZZLE_128B_ATOM_32B, the only MN-major layout
//   tcgen05 accepts for 32-bit operands). So x@W, dY@W^T and X^T@dY all run
//   without a transpose copy.
// * B may come from up to three tensors: segmented along N (fused QKV),
//   segmented along K (dX of fused QKV / SwiGLU), or paired along N (the
//   gate|up halves of a SwiGLU tile).
// * Epilogues: store (alpha, residual, accumulate), SwiGLU forward (writes
//   gate, up and silu(gate)*up), SwiGLU backward (dgate, dup from dh).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <type_traits>
#include "../common/sm100.cuh"

namespace abacus {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements = 128 bytes, one swizzle span

enum BMode : int { kBSingle = 0, kBSegN = 1, kBSegK = 2, kBDualN = 3 };
enum Epi : int { kEpiStore = 0, kEpiSwiGLU = 1, kEpiSwiGLUBwd = 2 };

struct alignas(64) Params {
  CUtensorMap tma_a;
  CUtensorMap tma_b[3];
  int M, N, K;       // N is the logical output width (hidden units for SwiGLU)
  int b_mode;
  int seg;           // segment length (elements) for kBSegN / kBSegK
  int num_n_tiles;
  float alpha;
  float* c;
  long long ldc;
  const float* r;    // residual added by the store epilogue (nullable)
  long long ldr;
  int accumulate;    // store epilogue: C += result
  // Split-K: work unit (tile, split y) covers k-tiles [y * k_tiles_per_split, ...)
  // and stores its fp32 partial at c + y * split_stride (reduced afterwards).
  int k_tiles_per_split;
  long long split_stride;
  // SwiGLU forward outputs (ld = ldh)
  float* g;
  float* u;
  float* h;
  long long ldh;
  // SwiGLU backward: inputs gate/up (ld = ld_gu) and output [dgate | dup] rows
  const float* g_in;
  const float* u_in;
  long long ld_gu;
  float* dgu;
  long long ld_dgu;
  // Batched mode: every operand map is 4-D (inner, rows, H, B); blockIdx.z =
  // b * batch_h + h selects the matrix, C is offset by b*c_stride_b + h*c_stride_h.
  int batched;
  int batch_h;
  long long c_stride_h, c_stride_b;
  // Grouped mode (batched with one matrix per expert, H = experts): the
  // row-indexed epilogue tensors (SwiGLU g / u / h, g_in / u_in / dgu, and the
  // row-map scatter meta) stack the experts' rows, z_rows rows per expert.
  long long z_rows;
  // Causal structure of attention-shaped products (square, queries = keys):
  //   1: skip tiles strictly above the diagonal (n0 >= m0 + BM), C untouched
  //   2: K range [0, m0 + BM)   (P @ V, dS @ K: keys after the last query)
  //   3: K range [m0, K)        (dS^T @ Q, P^T @ dO: queries before the first key)
  int causal;
  // Persistent schedule: gridDim.x CTAs loop over the tiles (never combined
  // with the gathered-operand waits below).
  int persistent;
  // Work units = tiles x splits x batch_z (split-K and batched matrices are
  // flattened into the persistent schedule, so every SM gets an equal share).
  int splits;
  int batch_z;
  // Tensor-parallel all-gather fused into the GEMM: the gathered operand
  // (A when wait_operand == 0, else B) holds rows pushed by the ranks that own
  // them, `wait_chunk` rows per rank inside every `wait_seq`-row sequence. A
  // CTA starts only once each owner of the rows it reads has published
  // `wait_epoch` in wait_flags[owner]; rows of this rank (wait_self) are local.
  const int* wait_flags;
  int wait_operand;
  int wait_epoch, wait_chunk, wait_seq, wait_self;
  // GEMM -> reduce-scatter: output row r is stored on rank (r % seq) / chunk,
  // into this rank's slot of that rank's staging buffer (scatter_base[owner]),
  // at row (r / seq) * chunk + r % chunk; every finished tile then adds 1 to
  // the owner's arrival counter for this rank (release, system scope).
  float* scatter_base[8];
  unsigned* scatter_counter[8];
  int scatter_chunk, scatter_seq;
  // Row-map scatter (expert parallel combine): with scatter_meta set, output
  // row r goes to rank meta[r] & 7 at row meta[r] >> 3 (not at all when
  // meta[r] < 0), and each tile adds to every destination's counter the
  // number of its rows that went there.
  const int* scatter_meta;
  int* status;
  // QK-norm + RoPE fused into the QKV projection (3xTF32 store epilogue of an
  // N-segmented [q | k | v] GEMM, qk_cols = H * head_dim columns per segment):
  // for the q and k tiles each row's heads are RMS-normalised over head_dim
  // (eps, gamma q_gamma / k_gamma), rotated (rotate-half pairs (i, i + hd/2),
  // cos / sin tables (P, hd/2) at position positions[row] or row % seq_len)
  // and stored to q_out / k_out (T, qk_cols); rstd[(row * 2 + which) * heads +
  // head] keeps 1 / rms for the backward. The raw projection is stored as usual.
  float* q_out;
  float* k_out;
  float* qk_rstd;
  const float* q_gamma;
  const float* k_gamma;
  const float* rope_cos;
  const float* rope_sin;
  const int64_t* positions;
  int seq_len, heads, head_dim, qk_cols;
  float qk_eps;
  // Optional phase trace: CTAs 0 and 1 stamp clock64 at
  // trace[(cta * 16 + slot) * 128 + i] for the first 128 k-tiles / chunks i:
  // 0 TMA issued, 1 converter saw the stage, 2 converter done, 3 MMA saw the
  // converted stage, 4 MMAs issued, 5 epilogue saw chunk i, 6 chunk i drained,
  // converter: 7 A split in registers, 8 A stored to TMEM (issued), 9 B lo
  // written, 10 TMEM stores complete.
  long long* trace;
};

// Wait (bounded) until every owner of stored rows [r0, r1) of the gathered
// operand has published the expected epoch.
__device__ __forceinline__ bool wait_gathered_rows(const Params& p, int r0, int r1) {
  unsigned done = 0;
  for (int r = r0; r < r1;) {
    const int pos = r % p.wait_seq;
    const int owner = pos / p.wait_chunk;
    if (owner != p.wait_self && !(done & (1u << owner))) {
      if (!wait_flag_geq(p.wait_flags + owner, p.wait_epoch, p.status)) return false;
      done |= 1u << owner;
    }
    r += p.wait_chunk - pos % p.wait_chunk;
  }
  return true;
}

template <int BN, bool A_MN, bool B_MN, int PASSES, int STAGES, bool PAIR = false>
struct Config {
  // CTA pair (cta_group::2, 3xTF32 only): the pair computes a 256 x BN tile;
  // each CTA holds its 128 rows of A and BN / 2 columns of B.
  static_assert(!PAIR || PASSES == 3, "CTA pairs are built for the 3xTF32 mode");
  static constexpr int kBCols = PAIR ? BN / 2 : BN;  // B columns in this CTA's shared memory
  static constexpr int kABytes = BM * BK * 4;
  static constexpr int kBBytes = kBCols * BK * 4;
  // 3xTF32 stage: A landing buffer, B hi (in place), B lo. A hi / lo live in
  // TMEM (written by the converter), so the MMA reads A without touching smem.
  static constexpr int kStageBytes = PASSES == 3 ? kABytes + 2 * kBBytes : kABytes + kBBytes;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 1024;
  // 3xTF32: warpgroup 0 = producer (warp 0) + MMA issuer (warp 1), warpgroup 1
  // = epilogue, warpgroups 2 and 3 = converters of the even / odd k-tiles
  // (two k-tiles are split at once: one converter's latency per k-tile is
  // longer than the k-tile's MMAs). 1 pass: warps 0, 1 and the epilogue 2-5.
  static constexpr int kThreads = PASSES == 3 ? 512 : 192;
  static constexpr int kEpiWarp0 = PASSES == 3 ? 4 : 2;
  static constexpr int kConvWarp0 = 8;
  // Register budgets after the split (3xTF32), per thread of each warpgroup:
  // 128 threads x (72 + 232 + 104 + 104) = 65536 = 512 threads x 128 at launch.
  static constexpr uint32_t kRegsCtrl = 72, kRegsEpi = 232, kRegsConv = 104;
  static_assert(PASSES != 3 || 128 * (kRegsCtrl + kRegsEpi + 2 * kRegsConv) == kThreads * 128,
                "warpgroup register budgets must add up to the launch's 65536");
  // 3xTF32 accumulates K in chunks of kChunk k-tiles into two alternating
  // TMEM buffers that the epilogue drains (see the epilogue).
  static constexpr bool kChunked = PASSES == 3;
  static constexpr int kChunk = 2;
  static constexpr int kATmem = 2 * BN;  // first TMEM column of the A stages (3xTF32)
  // A hi / lo stages in TMEM (3xTF32): at most 4 fit beside the two 128-column
  // accumulators, so shared-memory stages beyond that (CTA pairs: 6) are
  // recycled through their own release barriers.
  static constexpr int kAStages = STAGES < 4 ? STAGES : 4;
  // 1 pass: two accumulator buffers, so a persistent CTA's epilogue of one
  // tile overlaps the MMAs of the next.
  static constexpr int kAccCols = kChunked ? 2 * BN + kAStages * 2 * BK : 2 * BN;
  static constexpr uint32_t kTmemCols = kAccCols <= 32 ? 32 : (kAccCols <= 64 ? 64 : (kAccCols <= 128 ? 128 : (kAccCols <= 256 ? 256 : 512)));
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <int BN, bool A_MN, bool B_MN, int PASSES, int EPI, int STAGES, bool PAIR = false>
__global__ void __launch_bounds__(Config<BN, A_MN, B_MN, PASSES, STAGES, PAIR>::kThreads, 1)
    gemm_kernel(const __grid_constant__ Params p) {
  using Cfg = Config<BN, A_MN, B_MN, PASSES, STAGES, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[STAGES];
  __shared__ uint64_t empty_bar[STAGES];
  __shared__ uint64_t conv_bar[STAGES];
  __shared__ uint64_t accum_full[2];
  __shared__ uint64_t accum_empty[2];
  __shared__ uint64_t chunk_full[2];
  __shared__ uint64_t chunk_empty[2];
  __shared__ uint64_t a_empty[4];  // 3xTF32: TMEM A stage released by the MMAs
  __shared__ uint32_t tmem_base_slot;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
#define ABACUS_GEMM_TRACE(slot, i)                                                                   \
  if (p.trace != nullptr && blockIdx.x < 2 && (i) < 128) {                                           \
    p.trace[(blockIdx.x * 16 + (slot)) * 128 + (i)] = clock64();                                     \
  }
  // Abort early (uniformly for the whole CTA) if an earlier kernel on this
  // device already recorded an error.
  // (A pair never returns early: both CTAs must reach the pair TMEM
  // allocation and the closing cluster barrier; after an earlier error its
  // bounded waits end at once instead.)
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = *reinterpret_cast<volatile int*>(p.status);
  __syncthreads();
  if (!PAIR && abort_flag != kStatusOk) return;
  // Pair role: rank 0 issues the MMAs for both CTAs.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  // Shared-memory address of barrier `bar` in the pair's MMA-issuing CTA.
  auto leader_addr = [&](uint64_t* bar) { return mapa_shared(smem_u32(bar), 0); };

  // 1024-byte aligned stage buffers (swizzle period of SWIZZLE_128B).
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  auto stage_a = [&](int s) { return smem + s * Cfg::kStageBytes; };
  auto stage_b = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kABytes; };
  auto stage_blo = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes; };

  // Tile schedule. A persistent CTA (p.persistent) walks tiles blockIdx.x,
  // blockIdx.x + gridDim.x, ...; stage, chunk and accumulator phases run on
  // across tiles, so the epilogue of one tile overlaps the MMAs of the next.
  // Tiles are grouped along M for L2 reuse of B.
  // A pair walks 256-row tiles (rows [m0, m0 + 128) in rank 0, the next 128
  // in rank 1) with cluster index blockIdx.x / 2.
  constexpr int kTileM = PAIR ? 2 * BM : BM;
  const int num_m_tiles = (p.M + kTileM - 1) / kTileM;
  const int num_n_tiles = p.num_n_tiles;
  const int total_tiles = num_m_tiles * num_n_tiles;
  const int n_splits = max(1, p.splits);
  const int n_z = max(1, p.batch_z);
  const int total_units = total_tiles * n_splits * n_z;
  const int first_unit = PAIR ? static_cast<int>(blockIdx.x / 2) : static_cast<int>(blockIdx.x);
  const int unit_step = PAIR ? static_cast<int>(gridDim.x / 2) : (p.persistent ? static_cast<int>(gridDim.x) : total_units);
  constexpr int kGroup = 16;
  struct TileInfo {
    int m0, n0, kt_begin, num_k;
    int split, zh, zb;
    bool skip;
  };
  auto tile_at = [&](int unit) {
    TileInfo t;
    const int tile = unit % total_tiles;
    const int rest = unit / total_tiles;
    t.split = rest % n_splits;
    const int z = rest / n_splits;
    t.zh = p.batched ? z % p.batch_h : 0;
    t.zb = p.batched ? z / p.batch_h : 0;
    const int group = tile / (kGroup * num_n_tiles);
    const int first_m = group * kGroup;
    const int group_m = min(num_m_tiles - first_m, kGroup);
    const int in_group = tile - group * kGroup * num_n_tiles;
    t.m0 = (first_m + in_group % group_m) * kTileM + static_cast<int>(rank) * BM;
    // Output column base. For SwiGLU forward a tile covers BN/2 hidden units.
    t.n0 = (in_group / group_m) * (EPI == kEpiSwiGLU ? BN / 2 : BN);
    t.skip = p.causal == 1 && t.n0 >= t.m0 + BM;  // fully masked tile
    int total_k = (p.K + BK - 1) / BK;
    int kt_first = 0;
    if (p.causal == 2) total_k = min(total_k, (t.m0 + BM + BK - 1) / BK);
    if (p.causal == 3) kt_first = t.m0 / BK;
    t.kt_begin = kt_first + t.split * p.k_tiles_per_split;
    t.num_k = max(0, min(total_k, t.kt_begin + p.k_tiles_per_split) - t.kt_begin);
    return t;
  };
  if (!PAIR && !p.persistent && tile_at(blockIdx.x).skip) return;  // uniform exit
  int cur_h = 0, cur_b = 0;  // batched matrix of the tile being loaded (producer)
  if (!PAIR && p.wait_flags != nullptr) {
    // (Never persistent.) Rows of the gathered operand this CTA reads: the M
    // range for a K-major A, else the K range (MN-major A or B store tokens
    // along K).
    __shared__ int wait_ok;
    if (threadIdx.x == 0) {
      const TileInfo t = tile_at(blockIdx.x);
      if (p.wait_operand == 2) {
        // Rows pushed by every rank (expert-parallel dispatch): wait for all.
        bool good = true;
        for (int r = 0; r < p.wait_seq && good; ++r) {
          if (r != p.wait_self) good = wait_flag_geq(p.wait_flags + r, p.wait_epoch, p.status);
        }
        wait_ok = good ? 1 : 0;
      } else {
        const bool rows_are_m = p.wait_operand == 0 && !A_MN;
        const int r0 = rows_are_m ? t.m0 : t.kt_begin * BK;
        const int r1 = rows_are_m ? min(t.m0 + BM, p.M) : min((t.kt_begin + t.num_k) * BK, p.K);
        wait_ok = wait_gathered_rows(p, r0, r1) ? 1 : 0;
      }
    }
    __syncthreads();
    if (!wait_ok) return;
  }
  auto load = [&](void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    if (p.batched) tma_load_4d(dst, map, bar, x, y, cur_h, cur_b);
    else tma_load_2d(dst, map, bar, x, y);
  };

  // In a pair the converter and epilogue warps of both CTAs arrive once per
  // warp on the leader's conv_bar / chunk_empty (8 arrivals).
  constexpr uint32_t kWarpArrivals = PAIR ? 8 : 128;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], kWarpArrivals);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accum_full[b], 1);
      mbar_init(&accum_empty[b], 128);
      mbar_init(&chunk_full[b], 1);
      mbar_init(&chunk_empty[b], kWarpArrivals);
    }
    for (int s = 0; s < 4; ++s) mbar_init(&a_empty[s], 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tma_a);
    tma_prefetch_desc(&p.tma_b[0]);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&tmem_base_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&tmem_base_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  // A pair also needs the other CTA's barriers initialised before any remote
  // arrive: synchronise the whole cluster.
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;
  // Register split (3xTF32), at the top of each warpgroup's branch: the
  // epilogue holds 128 fp32 accumulators per thread, a converter a 32-element
  // hi / lo row, warpgroup 0 only control state.
  if (warp < Cfg::kEpiWarp0) {
  if constexpr (PASSES == 3) regs_decrease<Cfg::kRegsCtrl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      int issued = 0;  // k-tiles issued over all tiles of this CTA
      bool ok = true;
      for (int tile = first_unit; tile < total_units && ok; tile += unit_step) {
        const TileInfo t = tile_at(tile);
        if (t.skip) continue;
        const int m0 = t.m0, n0 = t.n0;
        cur_h = t.zh;
        cur_b = t.zb;
        for (int kt = 0; kt < t.num_k; ++kt) {
          const int s = issued % STAGES;
          const int use = issued / STAGES;
          if (use > 0 && !mbar_wait(&empty_bar[s], (use - 1) & 1, p.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int k0 = (t.kt_begin + kt) * BK;
          ABACUS_GEMM_TRACE(0, issued)
          mbar_arrive_expect_tx(&full_bar[s], Cfg::kABytes + Cfg::kBBytes);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 32; ++c) load(stage_a(s) + c * 32 * BK * 4, &p.tma_a, &full_bar[s], m0 + 32 * c, k0);
          } else {
            load(stage_a(s), &p.tma_a, &full_bar[s], k0, m0);
          }
          // B source for this (n, k) tile. A pair's CTA loads columns
          // [rank * BN / 2, (rank + 1) * BN / 2) of the tile; for the paired
          // gate|up tile that is the gate half in rank 0 and the up half in rank 1.
          const CUtensorMap* bmap = &p.tma_b[0];
          int bn = n0 + static_cast<int>(rank) * (BN / 2) * (PAIR && p.b_mode != kBDualN ? 1 : 0), bk = k0;
          if (p.b_mode == kBSegN) {
            const int sidx = bn / p.seg;
            bmap = &p.tma_b[sidx];
            bn = bn - sidx * p.seg;
          } else if (p.b_mode == kBSegK) {
            const int sidx = k0 / p.seg;
            bmap = &p.tma_b[sidx];
            bk = k0 - sidx * p.seg;
          }
          if (B_MN) {
            if (p.b_mode == kBDualN && PAIR) {
  #pragma unroll
              for (int c = 0; c < BN / 64; ++c)
                load(stage_b(s) + c * 32 * BK * 4, &p.tma_b[rank], &full_bar[s], n0 + 32 * c, k0);
            } else if (p.b_mode == kBDualN) {
  #pragma unroll
              for (int c = 0; c < BN / 64; ++c) {
                load(stage_b(s) + c * 32 * BK * 4, &p.tma_b[0], &full_bar[s], n0 + 32 * c, k0);
                load(stage_b(s) + (c + BN / 64) * 32 * BK * 4, &p.tma_b[1], &full_bar[s], n0 + 32 * c, k0);
              }
            } else {
  #pragma unroll
              for (int c = 0; c < Cfg::kBCols / 32; ++c)
                load(stage_b(s) + c * 32 * BK * 4, bmap, &full_bar[s], bn + 32 * c, bk);
            }
          } else {
            // K-major B boxes are kBCols rows (BN / 2 for the paired halves).
            if (p.b_mode == kBDualN && PAIR) {
              load(stage_b(s), &p.tma_b[rank], &full_bar[s], k0, n0);
            } else if (p.b_mode == kBDualN) {
              load(stage_b(s), &p.tma_b[0], &full_bar[s], k0, n0);
              load(stage_b(s) + (BN / 2) * BK * 4, &p.tma_b[1], &full_bar[s], k0, n0);
            } else {
              load(stage_b(s), bmap, &full_bar[s], bk, bn);
            }
          }
          ++issued;
        }
      }
      // Never leave a bulk copy in flight into a CTA that is about to exit.
      for (int it = max(0, issued - STAGES); it < issued; ++it) {
        mbar_wait(&full_bar[it % STAGES], (it / STAGES) & 1, nullptr, 0);
      }
      // In a pair, the leader's last commits also arrive here: let them land
      // before this CTA can leave.
      if (PAIR) {
        for (int it = max(0, issued - STAGES); it < issued; ++it) {
          if (!mbar_wait(&empty_bar[it % STAGES], (it / STAGES) & 1, p.status, kStatusTimeoutEmpty)) break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (In a pair only rank 0 issues; its MMAs span both CTAs.)
    if (leader && elect_one_sync()) {
      // 3xTF32 reads A from TMEM, which is always K-major (lane = row).
      constexpr uint32_t idesc = idesc_tf32(PAIR ? 2 * BM : BM, BN, PASSES == 3 ? false : A_MN, B_MN);
      auto wait_in = [&](uint64_t* bar, uint32_t parity, int code) { return mbar_wait(bar, parity, p.status, code); };
      // Commit to this barrier in every CTA of the pair.
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          mma_commit_pair(smem_u32(bar));
          mma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          mma_commit(bar);
        }
      };
      int it = 0;        // k-tiles consumed over all tiles
      int chunk0 = 0;    // K chunks issued before this tile (3xTF32)
      int tcount = 0;    // tiles accumulated (1 pass: TMEM buffer = tcount & 1)
      bool ok = true;
      for (int tile = first_unit; tile < total_units && ok; tile += unit_step) {
        const TileInfo t = tile_at(tile);
        if (t.skip) continue;
        const int num_k = t.num_k;
        const int abuf = tcount & 1;
        if (!Cfg::kChunked && tcount >= 2 &&
            !mbar_wait(&accum_empty[abuf], ((tcount >> 1) - 1) & 1, p.status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        bool issued_any = false;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          const int use = it / STAGES;
          const int chunk = chunk0 + kt / Cfg::kChunk;
          const int buf = Cfg::kChunked ? (chunk & 1) : abuf;
          const bool first_in_chunk = Cfg::kChunked ? (kt % Cfg::kChunk == 0) : (kt == 0);
          const bool last_in_chunk = Cfg::kChunked && (kt % Cfg::kChunk == Cfg::kChunk - 1 || kt == num_k - 1);
          if (Cfg::kChunked && first_in_chunk && chunk >= 2 &&
              !wait_in(&chunk_empty[buf], ((chunk >> 1) - 1) & 1, kStatusTimeoutAccum)) {
            ok = false;
            break;
          }
          uint64_t* ready = PASSES == 3 ? &conv_bar[s] : &full_bar[s];
          if (!wait_in(ready, use & 1, PASSES == 3 ? kStatusTimeoutConvert : kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          ABACUS_GEMM_TRACE(3, it)
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
          const uint32_t a_hi = smem_u32(stage_a(s));
          const uint32_t b_hi = smem_u32(stage_b(s));
  #pragma unroll
          for (int ks = 0; ks < BK / 8; ++ks) {
            // One MMA consumes K = 8 tf32 elements (32 bytes).
            const uint32_t a_off = A_MN ? ks * 8 * 128 : ks * 32;
            const uint32_t b_off = B_MN ? ks * 8 * 128 : ks * 32;
            auto desc_a = [&](uint32_t base) {
              return A_MN ? desc_mnmajor_sw128_32b(base + a_off, 32 * BK * 4) : desc_kmajor_sw128(base + a_off);
            };
            auto desc_b = [&](uint32_t base) {
              return B_MN ? desc_mnmajor_sw128_32b(base + b_off, 32 * BK * 4) : desc_kmajor_sw128(base + b_off);
            };
            const uint32_t acc = (first_in_chunk && ks == 0) ? 0u : 1u;
            if (PASSES == 3) {
              const uint32_t ta_hi = tmem_base + Cfg::kATmem + (it % Cfg::kAStages) * 2 * BK + ks * 8;
              const uint32_t ta_lo = ta_hi + BK;
              const uint32_t b_lo = smem_u32(stage_blo(s));
              if constexpr (PAIR) {
                mma_tf32_ts_pair(d_tmem, ta_lo, desc_b(b_hi), idesc, acc);
                mma_tf32_ts_pair(d_tmem, ta_hi, desc_b(b_lo), idesc, 1u);
                mma_tf32_ts_pair(d_tmem, ta_hi, desc_b(b_hi), idesc, 1u);
              } else {
                mma_tf32_ts(d_tmem, ta_lo, desc_b(b_hi), idesc, acc);
                mma_tf32_ts(d_tmem, ta_hi, desc_b(b_lo), idesc, 1u);
                mma_tf32_ts(d_tmem, ta_hi, desc_b(b_hi), idesc, 1u);
              }
            } else {
              mma_tf32_ss(d_tmem, desc_a(a_hi), desc_b(b_hi), idesc, acc);
            }
          }
          if (PASSES == 3 && Cfg::kAStages < STAGES) commit(&a_empty[it % Cfg::kAStages]);
          commit(&empty_bar[s]);
          if (last_in_chunk) commit(&chunk_full[buf]);
          ABACUS_GEMM_TRACE(4, it)
          issued_any = true;
        }
        if (!ok) break;
        if (Cfg::kChunked) {
          chunk0 += (num_k + Cfg::kChunk - 1) / Cfg::kChunk;
        } else {
          if (issued_any) mma_commit(&accum_full[abuf]);
          else mbar_arrive(&accum_full[abuf]);
          ++tcount;
        }
      }
      // Every commit must have landed before this CTA's shared memory is
      // released: wait for the last release of each stage (bounded).
      for (int j = max(0, it - STAGES); j < it; ++j) {
        if (!mbar_wait(&empty_bar[j % STAGES], (j / STAGES) & 1, p.status, kStatusTimeoutEmpty)) break;
      }
    }
  }  // warps 2 and 3 of warpgroup 0 (3xTF32) have no role
  } else if (warp >= Cfg::kEpiWarp0 && warp < Cfg::kEpiWarp0 + 4) {
    if constexpr (PASSES == 3) regs_increase<Cfg::kRegsEpi>();
    // ------------------------------------------------------------ epilogue
    const int q = warp % 4;  // TMEM lane quarter this warp may access
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    int chunk0 = 0, tcount = 0;
    bool dead = false;  // a wait ran out: skip all work, keep the named barriers
    for (int tile = first_unit; tile < total_units; tile += unit_step) {
      const TileInfo t = tile_at(tile);
      if (t.skip) continue;
      const int m0 = t.m0, n0 = t.n0, num_k = t.num_k;
      const int row = m0 + q * 32 + lane;
      // Row of the stacked (grouped) epilogue tensors.
      const long long grow = row + static_cast<long long>(t.zh) * p.z_rows;
      bool ok = num_k > 0 && !dead;
      const int abuf = tcount & 1;
      // fp32 (3xTF32) mode: drain each K-chunk accumulator into registers with
      // round-to-nearest fp32 adds, so the tensor core's own accumulation never
      // spans more than kChunk k-tiles.
      float acc[Cfg::kChunked ? BN : 1];
      if constexpr (Cfg::kChunked) {
#pragma unroll
        for (int i = 0; i < BN; ++i) acc[i] = 0.f;
        const int num_chunks = (num_k + Cfg::kChunk - 1) / Cfg::kChunk;
        for (int j = 0; j < num_chunks && ok; ++j) {
          const int c_idx = chunk0 + j;
          const int buf = c_idx & 1;
          if (!mbar_wait_warp(&chunk_full[buf], (c_idx >> 1) & 1, p.status, kStatusTimeoutAccum)) {
            ok = false;
            dead = true;
            break;
          }
          if (threadIdx.x == Cfg::kEpiWarp0 * 32) ABACUS_GEMM_TRACE(5, c_idx)
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(taddr + buf * BN + c * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[c * 32 + i] += __uint_as_float(v[i]);
          }
          tc_fence_before();
          if (threadIdx.x == Cfg::kEpiWarp0 * 32) ABACUS_GEMM_TRACE(6, c_idx)
          if constexpr (PAIR) {
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_addr(&chunk_empty[buf]));
          } else {
            mbar_arrive(&chunk_empty[buf]);
          }
        }
        chunk0 += num_chunks;
      } else {
        if (!dead) {
          if (!mbar_wait_warp(&accum_full[abuf], (tcount >> 1) & 1, p.status, kStatusTimeoutAccum)) {
            ok = false;
            dead = true;
          }
          tc_fence_after();
        }
      }
      // Fetch the 32 accumulator columns of group c.
      auto group = [&](int c, float (&out)[32]) {
        if constexpr (Cfg::kChunked) {
#pragma unroll
          for (int i = 0; i < 32; ++i) out[i] = acc[c * 32 + i];
        } else {
          uint32_t v[32];
          tmem_ld32(taddr + abuf * BN + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(v[i]);
        }
      };
      const bool row_ok = row < p.M;
      if (ok && EPI == kEpiStore) {
  #pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          group(c, v);
          const int col0 = n0 + c * 32;
          // Row-map scatter: rows whose meta is negative (unfilled capacity
          // slots of an expert slab) are computed but not returned.
          if (row_ok && col0 < p.N && (!p.scatter_meta || p.scatter_meta[grow] >= 0)) {
            float* crow;
            if (p.scatter_meta) {
              const int meta = p.scatter_meta[grow];
              crow = p.scatter_base[meta & 7] + static_cast<long long>(meta >> 3) * p.ldc + col0;
            } else if (p.scatter_chunk) {
              const int pos = row % p.scatter_seq;
              const int owner = pos / p.scatter_chunk;
              const long long lrow =
                  static_cast<long long>(row / p.scatter_seq) * p.scatter_chunk + (pos - owner * p.scatter_chunk);
              crow = p.scatter_base[owner] + lrow * p.ldc + col0;
            } else {
              crow = p.c + t.split * p.split_stride + t.zb * p.c_stride_b + t.zh * p.c_stride_h +
                     static_cast<long long>(row) * p.ldc + col0;
            }
            const float* rrow = p.r ? p.r + static_cast<long long>(row) * p.ldr + col0 : nullptr;
            if (col0 + 32 <= p.N) {
  #pragma unroll
              for (int j = 0; j < 32; j += 4) {
                float4 o = make_float4(v[j] * p.alpha, v[j + 1] * p.alpha, v[j + 2] * p.alpha, v[j + 3] * p.alpha);
                if (rrow) {
                  const float4 rv = *reinterpret_cast<const float4*>(rrow + j);
                  o.x += rv.x; o.y += rv.y; o.z += rv.z; o.w += rv.w;
                }
                if (p.accumulate) {
                  const float4 cv = *reinterpret_cast<const float4*>(crow + j);
                  o.x += cv.x; o.y += cv.y; o.z += cv.z; o.w += cv.w;
                }
                *reinterpret_cast<float4*>(crow + j) = o;
              }
            } else {
  #pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < p.N) {
                  float o = v[j] * p.alpha;
                  if (rrow) o += rrow[j];
                  if (p.accumulate) o += crow[j];
                  crow[j] = o;
                }
              }
            }
          }
        }
        if constexpr (Cfg::kChunked) {
          if (p.q_out != nullptr && row_ok && n0 < 2 * p.qk_cols) {
            // The tile's whole row is in acc: normalise and rotate its heads.
            const int which = n0 >= p.qk_cols ? 1 : 0;
            const long long pos = p.positions ? p.positions[row] : static_cast<long long>(row % p.seq_len);
            auto heads_of_row = [&](auto hd_c) {
              constexpr int HD = decltype(hd_c)::value, HALF = HD / 2;
              const float* gamma = which ? p.k_gamma : p.q_gamma;
              const float* cs = p.rope_cos + pos * HALF;
              const float* sn = p.rope_sin + pos * HALF;
#pragma unroll
              for (int j = 0; j < BN / HD; ++j) {
                float ss = 0.f;
#pragma unroll
                for (int i = 0; i < HD; ++i) ss = fmaf(acc[j * HD + i], acc[j * HD + i], ss);
                const float r = rsqrtf(ss / HD + p.qk_eps);
                const int head = (n0 - which * p.qk_cols) / HD + j;
                p.qk_rstd[(static_cast<long long>(row) * 2 + which) * p.heads + head] = r;
                float* dst = (which ? p.k_out : p.q_out) + static_cast<long long>(row) * p.qk_cols + head * HD;
#pragma unroll
                for (int i = 0; i < HALF; i += 4) {
                  const float4 c4 = *reinterpret_cast<const float4*>(cs + i);
                  const float4 s4 = *reinterpret_cast<const float4*>(sn + i);
                  const float4 g1 = *reinterpret_cast<const float4*>(gamma + i);
                  const float4 g2 = *reinterpret_cast<const float4*>(gamma + HALF + i);
                  const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
                  const float ga[4] = {g1.x, g1.y, g1.z, g1.w}, gb[4] = {g2.x, g2.y, g2.z, g2.w};
                  float o1[4], o2[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float n1 = ga[e] * acc[j * HD + i + e] * r;
                    const float n2 = gb[e] * acc[j * HD + HALF + i + e] * r;
                    o1[e] = n1 * cv[e] - n2 * sv[e];
                    o2[e] = n2 * cv[e] + n1 * sv[e];
                  }
                  *reinterpret_cast<float4*>(dst + i) = make_float4(o1[0], o1[1], o1[2], o1[3]);
                  *reinterpret_cast<float4*>(dst + HALF + i) = make_float4(o2[0], o2[1], o2[2], o2[3]);
                }
              }
            };
            if (p.head_dim == 64) heads_of_row(std::integral_constant<int, 64>{});
            else heads_of_row(std::integral_constant<int, 128>{});
          }
        }
      } else if (ok && EPI == kEpiSwiGLU) {
  #pragma unroll
        for (int c = 0; c < BN / 64; ++c) {
          float gv[32], uv[32];
          group(c, gv);
          group(c + BN / 64, uv);
          const int col0 = n0 + c * 32;
          if (row_ok && col0 < p.N) {
            const long long off = grow * p.ldh + col0;
            const bool vec = col0 + 32 <= p.N && (p.ldh & 3) == 0 &&
                             ((reinterpret_cast<uintptr_t>(p.g) | reinterpret_cast<uintptr_t>(p.u) |
                               reinterpret_cast<uintptr_t>(p.h)) & 15) == 0;
            if (vec) {
              // 16-byte stores: a quarter of the store instructions.
  #pragma unroll
              for (int j = 0; j < 32; j += 4) {
                *reinterpret_cast<float4*>(p.g + off + j) = make_float4(gv[j], gv[j + 1], gv[j + 2], gv[j + 3]);
                *reinterpret_cast<float4*>(p.u + off + j) = make_float4(uv[j], uv[j + 1], uv[j + 2], uv[j + 3]);
                *reinterpret_cast<float4*>(p.h + off + j) =
                    make_float4(silu_f(gv[j]) * uv[j], silu_f(gv[j + 1]) * uv[j + 1], silu_f(gv[j + 2]) * uv[j + 2],
                                silu_f(gv[j + 3]) * uv[j + 3]);
              }
            } else {
  #pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < p.N) {
                  p.g[off + j] = gv[j];
                  p.u[off + j] = uv[j];
                  p.h[off + j] = silu_f(gv[j]) * uv[j];
                }
              }
            }
          }
        }
      } else if (ok && EPI == kEpiSwiGLUBwd) {
  #pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          group(c, v);
          const int col0 = n0 + c * 32;
          if (row_ok && col0 < p.N) {
            const long long off = grow * p.ld_gu + col0;
            const long long doff = grow * p.ld_dgu + col0;
            const bool vec = col0 + 32 <= p.N && ((p.ld_gu | p.ld_dgu | p.N) & 3) == 0 &&
                             ((reinterpret_cast<uintptr_t>(p.g_in) | reinterpret_cast<uintptr_t>(p.u_in) |
                               reinterpret_cast<uintptr_t>(p.dgu)) & 15) == 0;
            if (vec) {
              // 16-byte loads and stores: a quarter of the memory instructions.
  #pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 g4 = *reinterpret_cast<const float4*>(p.g_in + off + j);
                const float4 u4 = *reinterpret_cast<const float4*>(p.u_in + off + j);
                const float gs[4] = {g4.x, g4.y, g4.z, g4.w}, us[4] = {u4.x, u4.y, u4.z, u4.w};
                float dg[4], du[4];
  #pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float dh = v[j + e];
                  const float sg = 1.0f / (1.0f + __expf(-gs[e]));
                  dg[e] = dh * us[e] * sg * (1.0f + gs[e] * (1.0f - sg));
                  du[e] = dh * gs[e] * sg;
                }
                *reinterpret_cast<float4*>(p.dgu + doff + j) = make_float4(dg[0], dg[1], dg[2], dg[3]);
                *reinterpret_cast<float4*>(p.dgu + doff + p.N + j) = make_float4(du[0], du[1], du[2], du[3]);
              }
            } else {
  #pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < p.N) {
                  const float dh = v[j];
                  const float g = p.g_in[off + j];
                  const float u = p.u_in[off + j];
                  const float sg = 1.0f / (1.0f + __expf(-g));
                  p.dgu[doff + j] = dh * u * sg * (1.0f + g * (1.0f - sg));
                  p.dgu[doff + p.N + j] = dh * g * sg;
                }
              }
            }
          }
        }
      }
      if (!Cfg::kChunked) {
        // The accumulator buffer may take the tile after next.
        if (!dead) {
          tc_fence_before();
          mbar_arrive(&accum_empty[abuf]);
        }
        ++tcount;
      }
      if (EPI == kEpiStore && p.scatter_chunk) {
        // Publish this tile to its owner once all four epilogue warps stored it.
        __shared__ int epi_ok[4];
        __threadfence_system();
        if (lane == 0) epi_ok[q] = ok ? 1 : 0;
        named_barrier_sync(1, 128);
        if (warp == Cfg::kEpiWarp0 && lane == 0 && epi_ok[0] && epi_ok[1] && epi_ok[2] && epi_ok[3]) {
          const int owner = (m0 % p.scatter_seq) / p.scatter_chunk;
          red_release_sys_add(p.scatter_counter[owner], 1u);
        }
      } else if (EPI == kEpiStore && p.scatter_meta) {
        // Count this tile's rows per destination rank, then publish them.
        __shared__ int epi_ok[4];
        __shared__ unsigned dest_rows[8];
        if (warp == Cfg::kEpiWarp0 && lane < 8) dest_rows[lane] = 0u;
        __threadfence_system();
        if (lane == 0) epi_ok[q] = ok ? 1 : 0;
        named_barrier_sync(1, 128);
        const int meta_row = row_ok ? p.scatter_meta[grow] : -1;
        const int dest = meta_row >= 0 ? (meta_row & 7) : -1;
  #pragma unroll
        for (int d = 0; d < 8; ++d) {
          const unsigned n = __popc(__ballot_sync(0xffffffffu, dest == d));
          if (lane == 0 && n) atomicAdd(&dest_rows[d], n);
        }
        named_barrier_sync(1, 128);
        if (warp == Cfg::kEpiWarp0 && lane == 0 && epi_ok[0] && epi_ok[1] && epi_ok[2] && epi_ok[3]) {
          for (int d = 0; d < 8; ++d)
            if (dest_rows[d]) red_release_sys_add(p.scatter_counter[d], dest_rows[d]);
        }
      }
    }
  } else if (PASSES == 3 && warp >= Cfg::kConvWarp0) {
    // ------------------------------------------------------------ converter
    // Thread = one row of the A tile (its TMEM lane): read the row from the
    // TMA landing buffer (undoing the swizzle), split it into tf32 hi / lo and
    // store both into this stage's TMEM columns. B is split in shared memory:
    // raw as hi, lo beside it. Converter group g takes the k-tiles with
    // it % 2 == g (with an even stage count, always the same stages).
    static_assert(STAGES % 2 == 0, "two converter groups alternate over the stages");
    regs_decrease<Cfg::kRegsConv>();
    const int group = (warp - Cfg::kConvWarp0) / 4;
    const int ct = threadIdx.x - Cfg::kConvWarp0 * 32 - group * 128;  // 0..127
    const bool tracer = ct == 0;
    const int row = (warp % 4) * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>((warp % 4) * 32) << 16);
    int it = 0;
    bool ok = true;
    for (int tile = first_unit; tile < total_units && ok; tile += unit_step) {
      const TileInfo t = tile_at(tile);
      if (t.skip) continue;
      for (int kt = 0; kt < t.num_k; ++kt, ++it) {
        if ((it & 1) != group) continue;
        const int s = it % STAGES;
        const int use = it / STAGES;
        if (!mbar_wait_warp(&full_bar[s], use & 1, p.status, kStatusTimeoutFull)) {
          ok = false;
          break;
        }
        if (tracer) ABACUS_GEMM_TRACE(1, it)
          const uint8_t* a = stage_a(s);
          uint32_t hi[BK], lo[BK];
          if (A_MN) {
            // [row / 32][k][128 B], 32-byte granules XOR-swizzled by (k & 3).
            const uint8_t* base = a + (row / 32) * 32 * BK * 4;
            const int b = (row % 32) * 4;
    #pragma unroll
            for (int k = 0; k < BK; ++k) {
              const int phys = (((b >> 5) ^ (k & 3)) << 5) | (b & 31);
              const float x = *reinterpret_cast<const float*>(base + k * 128 + phys);
              const float h = to_tf32(x);
              hi[k] = __float_as_uint(h);
              lo[k] = __float_as_uint(to_tf32_lo(x - h));
            }
          } else {
            // Row of 128 bytes, 16-byte chunks XOR-swizzled by (row & 7).
    #pragma unroll
            for (int c = 0; c < BK / 4; ++c) {
              const float4 x = *reinterpret_cast<const float4*>(a + row * 128 + ((c ^ (row & 7)) << 4));
              const float xs[4] = {x.x, x.y, x.z, x.w};
    #pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float h = to_tf32(xs[e]);
                hi[4 * c + e] = __float_as_uint(h);
                lo[4 * c + e] = __float_as_uint(to_tf32_lo(xs[e] - h));
              }
            }
          }
          // The TMEM A stage must have been read by the MMAs of k-tile
          // it - kAStages (with kAStages == STAGES that is already implied by
          // the TMA landing, which waited for the same MMAs).
          const int as = it % Cfg::kAStages;
          if (Cfg::kAStages < STAGES && it >= Cfg::kAStages &&
              !mbar_wait_warp(&a_empty[as], ((it / Cfg::kAStages) - 1) & 1, p.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (tracer) ABACUS_GEMM_TRACE(7, it)
          tc_fence_after();
          tmem_st32(lane_addr + Cfg::kATmem + as * 2 * BK, hi);
          tmem_st32(lane_addr + Cfg::kATmem + as * 2 * BK + BK, lo);
          if (tracer) ABACUS_GEMM_TRACE(8, it)
          // B stays raw in the landing buffer (the MMA truncates it to its tf32
          // hi part); only lo is written.
          const float4* bsrc = reinterpret_cast<const float4*>(stage_b(s));
          float4* bdst = reinterpret_cast<float4*>(stage_blo(s));
          constexpr int kB4 = Cfg::kBCols * BK / 4;
    #pragma unroll 4
          for (int i = ct; i < kB4; i += 128) {
            const float4 x = bsrc[i];
            bdst[i] = make_float4(tf32_lo_of_raw_alu(x.x), tf32_lo_of_raw_alu(x.y), tf32_lo_of_raw_alu(x.z),
                                   tf32_lo_of_raw_alu(x.w));
          }
          if (tracer) ABACUS_GEMM_TRACE(9, it)
          tmem_st_wait();
          if (tracer) ABACUS_GEMM_TRACE(10, it)
          fence_proxy_async_smem();
          tc_fence_before();
        if (tracer) ABACUS_GEMM_TRACE(2, it)
        if constexpr (PAIR) {
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_addr(&conv_bar[s]));
        } else {
          mbar_arrive(&conv_bar[s]);
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  // A pair waits for the whole cluster: the leader's MMAs read this CTA's
  // shared memory and TMEM until its last commit, which the leader's MMA
  // warp waited for above.
  tc_fence_before();
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace gemm
}  // namespace abacus
