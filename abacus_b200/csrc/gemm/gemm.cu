// Host side of the tcgen05 tf32 GEMM: tensor-map encoding, tile-config
// selection and the torch bindings used by abacus_b200.ops.linear.
#include <cstdlib>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include "gemm_launch.cuh"
#include "../common/host.h"
#include "../api.h"

namespace abacus {
namespace gemm {

namespace {

// 2-D fp32 tensor map over a row-major matrix with `rows` rows of `inner`
// elements and a row stride of `ld` elements; box = box_inner x box_rows.
CUtensorMap make_map(const float* base, int64_t inner, int64_t rows, int64_t ld, int box_inner, int box_rows,
                     bool mn_major) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = host::encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r), " (inner=", inner,
              " rows=", rows, " ld=", ld, ")");
  return m;
}

// Operand view: logical (rows_mn, k) matrix stored either K-major
// (row-major [mn][k]) or MN-major (row-major [k][mn]).
struct Operand {
  const float* ptr;
  int64_t mn, k, ld;
  bool mn_major;
};

Operand operand_of(const torch::Tensor& t, bool transposed_storage, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32, name, " must be a CUDA fp32 tensor");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit inner stride");
  TORCH_CHECK(t.stride(0) % 4 == 0 && t.stride(0) >= t.size(1), name,
              " row stride must be a multiple of 4 elements (16 bytes) for TMA");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned for TMA");
  Operand o;
  o.ptr = t.data_ptr<float>();
  o.ld = t.stride(0);
  o.mn_major = transposed_storage;
  if (transposed_storage) {  // stored [k][mn]
    o.k = t.size(0);
    o.mn = t.size(1);
  } else {  // stored [mn][k]
    o.mn = t.size(0);
    o.k = t.size(1);
  }
  return o;
}

CUtensorMap map_for(const Operand& o, int tile_mn) {
  if (o.mn_major) return make_map(o.ptr, o.mn, o.k, o.ld, 32, BK, true);
  return make_map(o.ptr, o.k, o.mn, o.ld, BK, tile_mn, false);
}

// C = alpha * sum_s ws[s] (+ residual) (+ C), summed in split order
// (deterministic). ws: (splits, M, N) contiguous.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, long long M, long long N, float alpha,
                                     const float* __restrict__ r, long long ldr, int accumulate, float* __restrict__ c,
                                     long long ldc) {
  const long long n4 = N / 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= M * n4) return;
  const long long m = idx / n4, j = (idx % n4) * 4;
  const long long plane = M * N;
  float4 acc = *reinterpret_cast<const float4*>(ws + m * N + j);
  for (int s = 1; s < splits; ++s) {
    const float4 v = *reinterpret_cast<const float4*>(ws + s * plane + m * N + j);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  acc.x *= alpha; acc.y *= alpha; acc.z *= alpha; acc.w *= alpha;
  if (r) {
    const float4 v = *reinterpret_cast<const float4*>(r + m * ldr + j);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  float* cp = c + m * ldc + j;
  if (accumulate) {
    const float4 v = *reinterpret_cast<const float4*>(cp);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  *reinterpret_cast<float4*>(cp) = acc;
}

// Number of K splits for a GEMM with `tiles` output tiles and `k_tiles`
// 32-deep k-tiles. Work units (tile, split) are shared evenly by one
// persistent CTA per SM, so pick the split count whose busiest SM does the
// fewest k-tiles, with at least 16 k-tiles per split; ties go to fewer splits
// (less reduction traffic).
int pick_splits(long long tiles, int k_tiles, int sms) {
  if (tiles >= 2LL * sms || k_tiles < 64) return 1;
  long long best_s = 1, best_cost = -1;
  for (long long s = 1; s <= 16 && k_tiles / s >= 16; ++s) {
    const long long per_unit = (k_tiles + s - 1) / s;
    const long long rounds = (tiles * s + sms - 1) / sms;
    const long long cost = rounds * per_unit;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_s = s;
    }
  }
  return static_cast<int>(best_s);
}

void check_passes(int64_t passes) { TORCH_CHECK(passes == 1 || passes == 3, "passes must be 1 (tf32) or 3 (3xTF32)"); }

// Grid width for `units` work units (tiles x splits x batched matrices):
// persistent (one CTA per SM) unless the CTAs wait for peer data, which must
// stay one unit per CTA.
unsigned tile_grid(Params& p, long long units, int device) {
  if (p.wait_flags != nullptr || units <= 0) {
    p.persistent = 0;
    return static_cast<unsigned>(std::max<long long>(units, 1));
  }
  const int sms = at::cuda::getDeviceProperties(device)->multiProcessorCount;
  p.persistent = 1;
  return static_cast<unsigned>(std::min<long long>(units, sms));
}

// 3xTF32 GEMMs with at least two 128-row tiles run on CTA pairs (cta_group::2:
// one MMA over 256 rows, each SM reads half of B), unless the launch waits for
// peer rows or scatters its output (those keep one tile per CTA).
// ABACUS_GEMM_PAIR=0 turns pairs off.
bool pair_enabled() {
  const char* e = std::getenv("ABACUS_GEMM_PAIR");
  return !(e != nullptr && e[0] == '0');
}

bool use_pair(int64_t passes, long long m, bool comm) { return pair_enabled() && passes == 3 && !comm && m >= 2 * BM; }

// Persistent grid of CTA pairs for `units` 256-row work units.
unsigned pair_grid(Params& p, long long units, int device) {
  const int sms = at::cuda::getDeviceProperties(device)->multiProcessorCount;
  p.persistent = 1;
  return static_cast<unsigned>(2 * std::max<long long>(1, std::min<long long>(units, sms / 2)));
}

// Tensor-parallel options of one GEMM launch (see Params in gemm_tcgen05.cuh).
//   wait    = [flags_ptr, operand (0 A / 1 B), epoch, chunk, seq, self]
//   scatter = [chunk, seq, base_0..base_{P-1}, counter_0..counter_{P-1}]
struct Comm {
  std::vector<int64_t> wait;
  std::vector<int64_t> scatter;
};

void apply_comm(Params& p, const Comm& cm, bool a_mn, bool b_mn) {
  if (!cm.wait.empty()) {
    TORCH_CHECK(cm.wait.size() == 6, "wait spec has 6 entries");
    TORCH_CHECK(cm.wait[3] > 0 && cm.wait[4] > 0 && cm.wait[4] % cm.wait[3] == 0, "bad gathered chunking");
    TORCH_CHECK(cm.wait[1] != 1 || b_mn, "a gathered B operand must store tokens along K (MN-major)");
    TORCH_CHECK(cm.wait[1] >= 0 && cm.wait[1] <= 2, "wait operand: 0 A rows, 1 B rows, 2 all ranks");
    TORCH_CHECK(cm.wait[1] != 2 || (cm.wait[4] >= 1 && cm.wait[4] <= 8), "all-ranks wait: seq = number of ranks");
    (void)a_mn;
    p.wait_flags = reinterpret_cast<const int*>(cm.wait[0]);
    p.wait_operand = static_cast<int>(cm.wait[1]);
    p.wait_epoch = static_cast<int>(cm.wait[2]);
    p.wait_chunk = static_cast<int>(cm.wait[3]);
    p.wait_seq = static_cast<int>(cm.wait[4]);
    p.wait_self = static_cast<int>(cm.wait[5]);
  }
  if (!cm.scatter.empty()) {
    TORCH_CHECK(cm.scatter.size() >= 4 && (cm.scatter.size() - 2) % 2 == 0, "bad scatter spec");
    const size_t world = (cm.scatter.size() - 2) / 2;
    TORCH_CHECK(world >= 1 && world <= 8, "scatter over 1..8 ranks");
    if (cm.scatter[0] == -1) {
      // Row-map mode: scatter[1] = device int32 meta per output row.
      TORCH_CHECK(cm.scatter[1] != 0 && cm.scatter[1] % 4 == 0, "row map pointer");
      p.scatter_meta = reinterpret_cast<const int*>(cm.scatter[1]);
    } else {
      TORCH_CHECK(cm.scatter[0] % BM == 0, "scatter chunk must be a multiple of ", BM, " rows");
      TORCH_CHECK(cm.scatter[1] == cm.scatter[0] * static_cast<int64_t>(world), "sequence = chunk * ranks");
      p.scatter_chunk = static_cast<int>(cm.scatter[0]);
      p.scatter_seq = static_cast<int>(cm.scatter[1]);
    }
    for (size_t i = 0; i < world; ++i) {
      TORCH_CHECK(cm.scatter[2 + i] % 16 == 0, "scatter destinations must be 16-byte aligned");
      p.scatter_base[i] = reinterpret_cast<float*>(cm.scatter[2 + i]);
      p.scatter_counter[i] = reinterpret_cast<unsigned*>(cm.scatter[2 + world + i]);
    }
  }
}

Comm make_comm(const c10::optional<std::vector<int64_t>>& wait, const c10::optional<std::vector<int64_t>>& scatter) {
  Comm c;
  if (wait) c.wait = *wait;
  if (scatter) c.scatter = *scatter;
  return c;
}

// Device pointers and sizes of the QK-norm + RoPE epilogue (Params::q_out ...).
struct QKFuse {
  float *q_out, *k_out, *rstd;
  const float *q_gamma, *k_gamma, *cos_t, *sin_t;
  int seq_len, heads, head_dim;
  float eps;
};

int64_t gemm_out_impl(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
                      int64_t b_mode, double alpha, c10::optional<torch::Tensor> residual, bool accumulate,
                      int64_t passes, const Comm& cm, const QKFuse* qk = nullptr);
void gemm_swiglu_impl(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                      torch::Tensor h, int64_t passes, const Comm& cm);
void gemm_swiglu_bwd_impl(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u, torch::Tensor dgu,
                          int64_t passes, const Comm& cm);

}  // namespace

// C = alpha * op(A) @ op(B) [+ residual] [+ C]
//   a: (M, K), or (K, M) when trans_a
//   b list: each (K, N_i) row-major, or (N_i, K) when trans_b
//   b_mode: 0 single, 1 segmented along N (C columns = concat of B_i),
//           2 segmented along K (A columns = concat of K_i)
void gemm_out(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
              int64_t b_mode, double alpha, c10::optional<torch::Tensor> residual, bool accumulate, int64_t passes) {
  (void)gemm_out_impl(c, a, bs, trans_a, trans_b, b_mode, alpha, residual, accumulate, passes, Comm{});
}

int64_t gemm_pair_clusters() { return last_pair_clusters(); }

// Phase trace of the following GEMM launches into buf (int64, >= 4096
// entries, see Params::trace); None turns it off.
void gemm_trace(c10::optional<torch::Tensor> buf) {
  if (!buf) {
    gemm_trace_buffer() = nullptr;
    return;
  }
  TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == torch::kInt64 && buf->is_contiguous() && buf->numel() >= 4096,
              "trace buffer: contiguous CUDA int64 with at least 4096 entries");
  gemm_trace_buffer() = reinterpret_cast<long long*>(buf->data_ptr<int64_t>());
}

// [q | k | v] = x @ [Wq | Wk | Wv] with QK-norm + RoPE in the epilogue:
// qkv (T, 3HK) raw, q / k (T, HK) normalised and rotated, rstd (T * 2 * H).
// gammas (head_dim,), cos / sin (P, head_dim / 2) with P > the positions used
// (row % seq_len).
void gemm_qkv_norm_rope(torch::Tensor qkv, torch::Tensor x, std::vector<torch::Tensor> ws, torch::Tensor q,
                        torch::Tensor k, torch::Tensor rstd, torch::Tensor q_gamma, torch::Tensor k_gamma,
                        torch::Tensor cos_t, torch::Tensor sin_t, int64_t seq_len, int64_t heads, int64_t head_dim,
                        double eps, int64_t passes) {
  const int64_t t = x.size(0), hk = heads * head_dim;
  for (auto* o : {&q, &k}) {
    TORCH_CHECK(o->is_cuda() && o->scalar_type() == torch::kFloat32 && o->is_contiguous() && o->size(0) == t &&
                    o->size(1) == hk && reinterpret_cast<uintptr_t>(o->data_ptr()) % 16 == 0,
                "q / k outputs: contiguous (T, heads * head_dim) fp32");
  }
  TORCH_CHECK(rstd.is_contiguous() && rstd.numel() == t * 2 * heads, "rstd: T * 2 * heads");
  for (auto* g : {&q_gamma, &k_gamma})
    TORCH_CHECK(g->is_contiguous() && g->numel() == head_dim && reinterpret_cast<uintptr_t>(g->data_ptr()) % 16 == 0,
                "gammas: contiguous (head_dim,)");
  for (auto* tb : {&cos_t, &sin_t})
    TORCH_CHECK(tb->is_contiguous() && tb->dim() == 2 && tb->size(1) == head_dim / 2 && tb->size(0) >= seq_len &&
                    reinterpret_cast<uintptr_t>(tb->data_ptr()) % 16 == 0,
                "cos / sin tables: contiguous (positions >= seq_len, head_dim / 2)");
  TORCH_CHECK(seq_len > 0, "seq_len");
  QKFuse f;
  f.q_out = q.data_ptr<float>();
  f.k_out = k.data_ptr<float>();
  f.rstd = rstd.data_ptr<float>();
  f.q_gamma = q_gamma.data_ptr<float>();
  f.k_gamma = k_gamma.data_ptr<float>();
  f.cos_t = cos_t.data_ptr<float>();
  f.sin_t = sin_t.data_ptr<float>();
  f.seq_len = static_cast<int>(seq_len);
  f.heads = static_cast<int>(heads);
  f.head_dim = static_cast<int>(head_dim);
  f.eps = static_cast<float>(eps);
  (void)gemm_out_impl(qkv, x, ws, false, false, kBSegN, 1.0, c10::nullopt, false, passes, Comm{}, &f);
}

// Number of N tiles a single-B GEMM of output width n uses (stores per row).
int64_t gemm_n_tiles(int64_t n, int64_t passes) {
  check_passes(passes);
  const int bn = pick_bn(n, static_cast<int>(passes));
  return (n + bn - 1) / bn;
}

// gemm_out with the tensor-parallel options: a gathered operand whose rows
// arrive from peers (wait) and/or an output scattered to the row owners'
// staging buffers (scatter; no residual / accumulate / split-K then).
// Returns the output tiles stored on each owner when scattering by chunks, the
// number of N tiles (stores per row) when scattering by row map, else 0.
int64_t gemm_out_tp(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
                    int64_t b_mode, double alpha, int64_t passes, c10::optional<std::vector<int64_t>> wait,
                    c10::optional<std::vector<int64_t>> scatter) {
  return gemm_out_impl(c, a, bs, trans_a, trans_b, b_mode, alpha, c10::nullopt, false, passes, make_comm(wait, scatter));
}

namespace {
int64_t gemm_out_impl(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
                      int64_t b_mode, double alpha, c10::optional<torch::Tensor> residual, bool accumulate,
                      int64_t passes, const Comm& cm, const QKFuse* qk) {
  check_passes(passes);
  TORCH_CHECK(!bs.empty() && bs.size() <= 3, "between 1 and 3 B operands");
  const c10::cuda::CUDAGuard guard(a.device());
  Operand A = operand_of(a, trans_a, "A");
  std::vector<Operand> B;
  for (auto& b : bs) B.push_back(operand_of(b, !trans_b, "B"));
  int64_t M = A.mn, K = A.k, N = 0, seg = 0;
  if (b_mode == kBSingle) {
    TORCH_CHECK(bs.size() == 1);
    N = B[0].mn;
    TORCH_CHECK(B[0].k == K, "inner dimensions differ: ", K, " vs ", B[0].k);
  } else if (b_mode == kBSegN) {
    seg = B[0].mn;
    for (auto& o : B) TORCH_CHECK(o.mn == seg && o.k == K, "segmented-N operands must share shape");
    N = seg * static_cast<int64_t>(B.size());
  } else if (b_mode == kBSegK) {
    seg = B[0].k;
    N = B[0].mn;
    for (auto& o : B) TORCH_CHECK(o.k == seg && o.mn == N, "segmented-K operands must share shape");
    TORCH_CHECK(K == seg * static_cast<int64_t>(B.size()), "A width must equal the sum of the K segments");
  } else {
    TORCH_CHECK(false, "bad b_mode");
  }
  TORCH_CHECK(c.is_cuda() && c.scalar_type() == torch::kFloat32 && c.dim() == 2 && c.stride(1) == 1, "bad C");
  const bool scatter = !cm.scatter.empty();
  if (scatter) {
    // C is this rank's staging slice (M / ranks, N): it only fixes the row stride.
    TORCH_CHECK(c.size(1) == N && c.stride(0) == N, "scatter staging rows must be (.., N) contiguous");
    TORCH_CHECK(!residual && !accumulate, "scatter GEMMs take no residual / accumulate");
  } else {
    TORCH_CHECK(c.size(0) == M && c.size(1) == N, "C shape mismatch");
  }
  TORCH_CHECK(c.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0, "C must be 16-byte aligned rows");
  if (M == 0 || N == 0) return 0;
  if (K == 0) {
    if (!accumulate) c.zero_();
    if (residual) c.add_(*residual);
    return 0;
  }
  int BN = pick_bn(N, static_cast<int>(passes));
  if (b_mode == kBSegN && seg % BN != 0) BN = 128;
  if (b_mode == kBSegN) TORCH_CHECK(seg % BN == 0, "segment width ", seg, " must be a multiple of the N tile ", BN);
  if (b_mode == kBSegK) TORCH_CHECK(seg % BK == 0, "segment depth must be a multiple of ", BK);
  const bool pair = use_pair(passes, M, !cm.wait.empty() || scatter);
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = map_for(A, BM);
  for (size_t i = 0; i < B.size(); ++i) p.tma_b[i] = map_for(B[i], pair ? BN / 2 : BN);
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.b_mode = static_cast<int>(b_mode);
  p.seg = static_cast<int>(seg);
  p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.alpha = static_cast<float>(alpha);
  p.c = c.data_ptr<float>();
  p.ldc = c.stride(0);
  if (residual) {
    TORCH_CHECK(residual->sizes() == c.sizes() && residual->stride(1) == 1 && residual->stride(0) % 4 == 0, "bad residual");
    p.r = residual->data_ptr<float>();
    p.ldr = residual->stride(0);
  }
  p.accumulate = accumulate ? 1 : 0;
  p.status = host::status_ptr(a.device().index());
  apply_comm(p, cm, A.mn_major, B[0].mn_major);
  if (qk != nullptr) {
    TORCH_CHECK(passes == 3 && b_mode == kBSegN && bs.size() == 3 && BN == 128 && seg % BN == 0, "fused QK-norm "
                "+ RoPE needs the 3xTF32 N-segmented [q | k | v] GEMM with 128-column segments");
    TORCH_CHECK(qk->head_dim == 64 || qk->head_dim == 128, "fused QK-norm + RoPE: head_dim 64 or 128");
    TORCH_CHECK(!residual && !accumulate && alpha == 1.0 && cm.wait.empty() && cm.scatter.empty(),
                "fused QK-norm + RoPE takes a plain store");
    TORCH_CHECK(seg == static_cast<int64_t>(qk->heads) * qk->head_dim, "segment width must be heads * head_dim");
    p.q_out = qk->q_out;
    p.k_out = qk->k_out;
    p.qk_rstd = qk->rstd;
    p.q_gamma = qk->q_gamma;
    p.k_gamma = qk->k_gamma;
    p.rope_cos = qk->cos_t;
    p.rope_sin = qk->sin_t;
    p.seq_len = qk->seq_len;
    p.heads = qk->heads;
    p.head_dim = qk->head_dim;
    p.qk_cols = static_cast<int>(seg);
    p.qk_eps = qk->eps;
  }
  const long long tiles = ((M + BM - 1) / BM) * p.num_n_tiles;
  // Work units: 128-row tiles, or 256-row tiles of a CTA pair.
  const long long units = pair ? ((M + 2 * BM - 1) / (2 * BM)) * p.num_n_tiles : tiles;
  const int k_tiles = static_cast<int>((K + BK - 1) / BK);
  const int sms = at::cuda::getDeviceProperties(a.device().index())->multiProcessorCount;
  int splits = (N % 4 == 0 && !scatter && qk == nullptr) ? pick_splits(units, k_tiles, pair ? sms / 2 : sms) : 1;
  auto stream = at::cuda::getCurrentCUDAStream();
  p.k_tiles_per_split = (k_tiles + splits - 1) / splits;
  splits = (k_tiles + p.k_tiles_per_split - 1) / p.k_tiles_per_split;
  if (splits == 1) {
    p.splits = 1;
    p.batch_z = 1;
    const unsigned gx = pair ? pair_grid(p, units, a.device().index()) : tile_grid(p, tiles, a.device().index());
    launch_store(p, dim3(gx, 1), BN, A.mn_major, B[0].mn_major, static_cast<int>(passes), stream, pair);
    if (!scatter) return 0;
    if (cm.scatter[0] == -1) return p.num_n_tiles;  // each row lands once per N tile
    const int64_t owners = (static_cast<int64_t>(cm.scatter.size()) - 2) / 2;
    TORCH_CHECK(M % (static_cast<int64_t>(BM) * owners) == 0, "scattered rows must split evenly into tiles per owner");
    return (M / BM / owners) * p.num_n_tiles;
  }
  // Split-K: partials into a workspace, then one deterministic reduction that
  // also applies alpha / residual / accumulate.
  auto ws = torch::empty({splits, M, N}, c.options());
  Params q = p;
  q.c = ws.data_ptr<float>();
  q.ldc = N;
  q.split_stride = M * N;
  q.alpha = 1.f;
  q.r = nullptr;
  q.accumulate = 0;
  q.splits = splits;
  q.batch_z = 1;
  const unsigned gxs = pair ? pair_grid(q, units * splits, a.device().index())
                           : tile_grid(q, tiles * splits, a.device().index());
  launch_store(q, dim3(gxs, 1), BN, A.mn_major, B[0].mn_major, static_cast<int>(passes), stream, pair);
  const long long items = M * (N / 4);
  splitk_reduce_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(
      ws.data_ptr<float>(), splits, M, N, p.alpha, p.r, p.ldr, p.accumulate, p.c, p.ldc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  return 0;
}
}  // namespace

namespace {

// 4-D fp32 tensor map over a (B, H, rows, inner) strided view.
CUtensorMap make_map4(const torch::Tensor& t, int box_inner, int box_rows, bool mn_major) {
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(t.size(3)), static_cast<cuuint64_t>(t.size(2)),
                        static_cast<cuuint64_t>(t.size(1)), static_cast<cuuint64_t>(t.size(0))};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.stride(2) * 4), static_cast<cuuint64_t>(t.stride(1) * 4),
                           static_cast<cuuint64_t>(t.stride(0) * 4)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw = mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = host::encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, t.data_ptr(), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (4-D) failed with code ", static_cast<int>(r));
  return m;
}

void check_batched(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.dim() == 4, name,
              " must be a 4-D (B, H, rows, cols) CUDA fp32 view");
  TORCH_CHECK(t.stride(3) == 1, name, " must have unit inner stride");
  for (int d = 0; d < 3; ++d)
    TORCH_CHECK(t.stride(d) % 4 == 0, name, " strides must be multiples of 4 elements (16 bytes) for TMA");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned for TMA");
}

}  // namespace

// Batched C[b, h] = alpha * op(A[b, h]) @ op(B[b, h]) over (B, H, rows, cols)
// strided views (heads of a packed projection need no copy). `causal` selects
// the attention-shaped tile skipping described in gemm_tcgen05.cuh.
void gemm_batched(torch::Tensor c, torch::Tensor a, torch::Tensor b, bool trans_a, bool trans_b, double alpha,
                  int64_t causal, int64_t passes) {
  check_passes(passes);
  const c10::cuda::CUDAGuard guard(a.device());
  check_batched(a, "A");
  check_batched(b, "B");
  check_batched(c, "C");
  TORCH_CHECK(a.size(0) == b.size(0) && a.size(1) == b.size(1) && c.size(0) == a.size(0) && c.size(1) == a.size(1),
              "batch dimensions differ");
  const bool a_mn = trans_a, b_mn = !trans_b;
  const int64_t M = a_mn ? a.size(3) : a.size(2), K = a_mn ? a.size(2) : a.size(3);
  const int64_t N = b_mn ? b.size(3) : b.size(2), Kb = b_mn ? b.size(2) : b.size(3);
  TORCH_CHECK(K == Kb, "inner dimensions differ: ", K, " vs ", Kb);
  TORCH_CHECK(c.size(2) == M && c.size(3) == N, "C shape mismatch");
  TORCH_CHECK(causal >= 0 && causal <= 3, "causal mode must be 0..3");
  TORCH_CHECK(causal == 0 || (M == K || causal == 1), "causal modes 2/3 need a square (queries x keys) operand");
  const int64_t Z = a.size(0) * a.size(1);
  if (M == 0 || N == 0 || Z == 0) return;
  TORCH_CHECK(K > 0, "empty inner dimension");
  TORCH_CHECK(Z <= 65535, "at most 65535 matrices per batched GEMM");
  const int BN = pick_bn(N, static_cast<int>(passes));
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = a_mn ? make_map4(a, 32, BK, true) : make_map4(a, BK, BM, false);
  p.tma_b[0] = b_mn ? make_map4(b, 32, BK, true) : make_map4(b, BK, BN, false);
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.b_mode = kBSingle;
  p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.alpha = static_cast<float>(alpha);
  p.c = c.data_ptr<float>();
  p.ldc = c.stride(2);
  p.batched = 1;
  p.batch_h = static_cast<int>(a.size(1));
  p.c_stride_h = c.stride(1);
  p.c_stride_b = c.stride(0);
  p.causal = static_cast<int>(causal);
  p.status = host::status_ptr(a.device().index());
  p.k_tiles_per_split = static_cast<int>((K + BK - 1) / BK);
  const long long tiles = ((M + BM - 1) / BM) * p.num_n_tiles;
  p.splits = 1;
  p.batch_z = static_cast<int>(Z);
  const unsigned gxb = tile_grid(p, tiles * Z, a.device().index());
  launch_store(p, dim3(gxb, 1, 1), BN, a_mn, b_mn,
               static_cast<int>(passes), at::cuda::getCurrentCUDAStream());
}

// ------------------------------------------------------------ grouped GEMMs
// One launch over E experts: every operand is a 3-D (E, rows, cols) view
// (expert e's matrix at index e), mapped as a 4-D (1, E, rows, cols) TMA
// tensor; the tile schedule walks (tile, expert) units. Epilogue tensors that
// are indexed by row (SwiGLU outputs, the row-map scatter meta) stack the
// experts' rows: expert e's row r is row e * rows + r.
namespace {

torch::Tensor as4(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 3, name, " must be a 3-D (experts, rows, cols) view");
  return t.unsqueeze(0);
}

// Rows of a stacked 3-D view (stride(0) == rows * stride(1)), for the
// row-indexed epilogue tensors.
void check_stacked(const torch::Tensor& t, int64_t rows, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.dim() == 3 && t.stride(2) == 1, name,
              " must be a 3-D CUDA fp32 view with unit inner stride");
  TORCH_CHECK(t.size(1) == rows && t.stride(0) == rows * t.stride(1), name, " must stack ", rows, " rows per expert");
}

}  // namespace

// C[e] = alpha * op(A[e]) @ op(B[e]) (+ C[e]) for every expert e, one launch.
// b_mode 0 (single) or 2 (K-segmented: A's columns are the concatenation of
// the segments' K ranges). scatter: row-map mode only ([-1, meta, bases...,
// counters...]; meta indexed by stacked output row), C then only fixes the row
// stride.
int64_t gemm_grouped(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
                     int64_t b_mode, double alpha, bool accumulate, int64_t passes,
                     c10::optional<std::vector<int64_t>> scatter) {
  check_passes(passes);
  TORCH_CHECK(!bs.empty() && bs.size() <= 3, "between 1 and 3 B operands");
  TORCH_CHECK(b_mode == kBSingle || b_mode == kBSegK, "grouped GEMMs take a single or K-segmented B");
  const c10::cuda::CUDAGuard guard(a.device());
  auto a4 = as4(a, "A");
  check_batched(a4, "A");
  std::vector<torch::Tensor> b4;
  for (auto& b : bs) {
    b4.push_back(as4(b, "B"));
    check_batched(b4.back(), "B");
    TORCH_CHECK(b.size(0) == a.size(0), "every operand needs one matrix per expert");
  }
  const int64_t E = a.size(0);
  const bool a_mn = trans_a, b_mn = !trans_b;
  const int64_t M = a_mn ? a.size(2) : a.size(1), K = a_mn ? a.size(1) : a.size(2);
  const int64_t N = b_mn ? bs[0].size(2) : bs[0].size(1);
  const int64_t seg = b_mn ? bs[0].size(1) : bs[0].size(2);
  for (auto& b : bs) TORCH_CHECK((b_mn ? b.size(2) : b.size(1)) == N && (b_mn ? b.size(1) : b.size(2)) == seg, "B shapes differ");
  if (b_mode == kBSingle) {
    TORCH_CHECK(bs.size() == 1 && seg == K, "inner dimensions differ: ", K, " vs ", seg);
  } else {
    TORCH_CHECK(seg % BK == 0 && K == seg * static_cast<int64_t>(bs.size()), "K segments must be whole k-tiles summing to K");
  }
  const Comm cm = make_comm(c10::nullopt, scatter);
  const bool scattered = !cm.scatter.empty();
  TORCH_CHECK(!scattered || cm.scatter[0] == -1, "grouped GEMMs scatter by row map only");
  TORCH_CHECK(!scattered || !accumulate, "scatter GEMMs do not accumulate");
  auto c4 = as4(c, "C");
  if (!scattered) {
    check_batched(c4, "C");
    TORCH_CHECK(c.size(0) == E && c.size(1) == M && c.size(2) == N, "C shape mismatch");
  } else {
    TORCH_CHECK(c.stride(2) == 1 && c.size(2) == N && c.stride(1) == N, "scatter staging rows must be (.., N) contiguous");
  }
  if (M == 0 || N == 0 || E == 0) return 0;
  TORCH_CHECK(K > 0, "empty inner dimension");
  TORCH_CHECK(E <= 65535, "at most 65535 experts per grouped GEMM");
  const int BN = pick_bn(N, static_cast<int>(passes));
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = a_mn ? make_map4(a4, 32, BK, true) : make_map4(a4, BK, BM, false);
  for (size_t i = 0; i < b4.size(); ++i) p.tma_b[i] = b_mn ? make_map4(b4[i], 32, BK, true) : make_map4(b4[i], BK, BN, false);
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.b_mode = static_cast<int>(b_mode);
  p.seg = static_cast<int>(seg);
  p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.alpha = static_cast<float>(alpha);
  p.accumulate = accumulate ? 1 : 0;
  p.c = c.data_ptr<float>();
  p.ldc = c.stride(1);
  p.batched = 1;
  p.batch_h = static_cast<int>(E);
  p.c_stride_h = c.stride(0);
  p.z_rows = M;
  p.status = host::status_ptr(a.device().index());
  apply_comm(p, cm, a_mn, b_mn);
  p.k_tiles_per_split = static_cast<int>((K + BK - 1) / BK);
  const long long tiles = ((M + BM - 1) / BM) * p.num_n_tiles;
  p.splits = 1;
  p.batch_z = static_cast<int>(E);
  const unsigned grid = tile_grid(p, tiles * E, a.device().index());
  launch_store(p, dim3(grid, 1, 1), BN, a_mn, b_mn, static_cast<int>(passes), at::cuda::getCurrentCUDAStream());
  return scattered ? p.num_n_tiles : 0;
}

// Grouped SwiGLU up-projection: for every expert e, g[e] = x[e] @ w_gate[e],
// u[e] = x[e] @ w_up[e], h[e] = silu(g[e]) * u[e]. x (E, C, D); w (E, D, Mh);
// g / u / h (E, C, Mh) stacked. wait: as gemm_swiglu_tp (x rows pushed by peers).
void gemm_swiglu_grouped(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                         torch::Tensor h, int64_t passes, c10::optional<std::vector<int64_t>> wait) {
  check_passes(passes);
  const c10::cuda::CUDAGuard guard(x.device());
  auto x4 = as4(x, "x"), wg4 = as4(w_gate, "w_gate"), wu4 = as4(w_up, "w_up");
  check_batched(x4, "x");
  check_batched(wg4, "w_gate");
  check_batched(wu4, "w_up");
  const int64_t E = x.size(0), C = x.size(1), D = x.size(2), Mh = w_gate.size(2);
  TORCH_CHECK(w_gate.size(0) == E && w_up.size(0) == E && w_gate.size(1) == D && w_up.sizes() == w_gate.sizes(),
              "grouped SwiGLU weight shapes");
  for (auto* t : {&g, &u, &h}) check_stacked(*t, C, "SwiGLU output");
  TORCH_CHECK(g.stride(1) == h.stride(1) && u.stride(1) == h.stride(1) && g.size(2) == Mh && u.size(2) == Mh &&
                  h.size(2) == Mh && g.size(0) == E,
              "SwiGLU outputs must share (E, C, hidden) shape and row stride");
  if (E == 0 || C == 0 || Mh == 0) return;
  const int BN = passes == 3 ? 128 : 256;
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = make_map4(x4, BK, BM, false);
  p.tma_b[0] = make_map4(wg4, 32, BK, true);
  p.tma_b[1] = make_map4(wu4, 32, BK, true);
  p.M = static_cast<int>(C);
  p.N = static_cast<int>(Mh);
  p.K = static_cast<int>(D);
  p.b_mode = kBDualN;
  p.num_n_tiles = static_cast<int>((Mh + BN / 2 - 1) / (BN / 2));
  p.alpha = 1.f;
  p.g = g.data_ptr<float>();
  p.u = u.data_ptr<float>();
  p.h = h.data_ptr<float>();
  p.ldh = h.stride(1);
  p.batched = 1;
  p.batch_h = static_cast<int>(E);
  p.z_rows = C;
  p.status = host::status_ptr(x.device().index());
  apply_comm(p, make_comm(wait, c10::nullopt), false, true);
  p.k_tiles_per_split = static_cast<int>((D + BK - 1) / BK);
  const long long tiles = ((C + BM - 1) / BM) * p.num_n_tiles;
  p.splits = 1;
  p.batch_z = static_cast<int>(E);
  const unsigned grid = tile_grid(p, tiles * E, x.device().index());
  launch_swiglu(p, dim3(grid, 1), BN, static_cast<int>(passes), at::cuda::getCurrentCUDAStream());
}

// Grouped SwiGLU backward through the hidden layer: dh[e] = dy[e] @ w_down[e]^T,
// dgu[e] = [dh * u * silu'(g) | dh * silu(g)]. dy (E, C, D); w_down (E, Mh, D);
// g / u (E, C, Mh) and dgu (E, C, 2 Mh) stacked.
void gemm_swiglu_bwd_grouped(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u,
                             torch::Tensor dgu, int64_t passes, c10::optional<std::vector<int64_t>> wait) {
  check_passes(passes);
  const c10::cuda::CUDAGuard guard(dy.device());
  auto dy4 = as4(dy, "dy"), wd4 = as4(w_down, "w_down");
  check_batched(dy4, "dy");
  check_batched(wd4, "w_down");
  const int64_t E = dy.size(0), C = dy.size(1), D = dy.size(2), Mh = w_down.size(1);
  TORCH_CHECK(w_down.size(0) == E && w_down.size(2) == D, "w_down shape");
  check_stacked(g, C, "g");
  check_stacked(u, C, "u");
  check_stacked(dgu, C, "dgu");
  TORCH_CHECK(g.size(2) == Mh && u.sizes() == g.sizes() && u.stride(1) == g.stride(1) && dgu.size(2) == 2 * Mh,
              "g / u (E, C, hidden), dgu (E, C, 2 hidden)");
  if (E == 0 || C == 0 || Mh == 0) return;
  const int BN = passes == 3 ? 128 : (Mh >= 2048 ? 256 : 128);
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = make_map4(dy4, BK, BM, false);
  p.tma_b[0] = make_map4(wd4, BK, BN, false);
  p.M = static_cast<int>(C);
  p.N = static_cast<int>(Mh);
  p.K = static_cast<int>(D);
  p.b_mode = kBSingle;
  p.num_n_tiles = static_cast<int>((Mh + BN - 1) / BN);
  p.alpha = 1.f;
  p.g_in = g.data_ptr<float>();
  p.u_in = u.data_ptr<float>();
  p.ld_gu = g.stride(1);
  p.dgu = dgu.data_ptr<float>();
  p.ld_dgu = dgu.stride(1);
  p.batched = 1;
  p.batch_h = static_cast<int>(E);
  p.z_rows = C;
  p.status = host::status_ptr(dy.device().index());
  apply_comm(p, make_comm(wait, c10::nullopt), false, false);
  p.k_tiles_per_split = static_cast<int>((D + BK - 1) / BK);
  const long long tiles = ((C + BM - 1) / BM) * p.num_n_tiles;
  p.splits = 1;
  p.batch_z = static_cast<int>(E);
  const unsigned grid = tile_grid(p, tiles * E, dy.device().index());
  launch_swiglu_bwd(p, dim3(grid, 1), BN, static_cast<int>(passes), at::cuda::getCurrentCUDAStream());
}

// SwiGLU up-projection: g = x @ w_gate, u = x @ w_up, h = silu(g) * u.
// x (T, D), w_gate / w_up (D, Mh) in the (in, out) layout.
void gemm_swiglu(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                 torch::Tensor h, int64_t passes) {
  gemm_swiglu_impl(x, w_gate, w_up, g, u, h, passes, Comm{});
}

void gemm_swiglu_tp(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                    torch::Tensor h, int64_t passes, std::vector<int64_t> wait) {
  gemm_swiglu_impl(x, w_gate, w_up, g, u, h, passes, make_comm(wait, c10::nullopt));
}

namespace {
void gemm_swiglu_impl(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                      torch::Tensor h, int64_t passes, const Comm& cm) {
  check_passes(passes);
  const c10::cuda::CUDAGuard guard(x.device());
  Operand A = operand_of(x, false, "x");
  Operand Bg = operand_of(w_gate, true, "w_gate");
  Operand Bu = operand_of(w_up, true, "w_up");
  TORCH_CHECK(Bg.k == A.k && Bu.k == A.k && Bg.mn == Bu.mn, "SwiGLU shapes");
  const int64_t T = A.mn, Mh = Bg.mn;
  for (auto* t : {&g, &u, &h}) {
    TORCH_CHECK(t->size(0) == T && t->size(1) == Mh && t->stride(1) == 1 && t->stride(0) == h.stride(0),
                "SwiGLU outputs must be (T, hidden) with a shared row stride");
  }
  if (T == 0 || Mh == 0) return;
  const int BN = passes == 3 ? 128 : 256;
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = map_for(A, BM);
  p.tma_b[0] = map_for(Bg, BN / 2);
  p.tma_b[1] = map_for(Bu, BN / 2);
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(Mh);
  p.K = static_cast<int>(A.k);
  p.b_mode = kBDualN;
  p.num_n_tiles = static_cast<int>((Mh + BN / 2 - 1) / (BN / 2));
  p.alpha = 1.f;
  p.g = g.data_ptr<float>();
  p.u = u.data_ptr<float>();
  p.h = h.data_ptr<float>();
  p.ldh = h.stride(0);
  p.status = host::status_ptr(x.device().index());
  apply_comm(p, cm, false, true);
  p.k_tiles_per_split = static_cast<int>((A.k + BK - 1) / BK);
  const bool pair = use_pair(passes, T, !cm.wait.empty());
  const long long tiles = ((T + BM - 1) / BM) * p.num_n_tiles;
  const long long units = ((T + 2 * BM - 1) / (2 * BM)) * p.num_n_tiles;
  p.splits = 1;
  p.batch_z = 1;
  const unsigned grid = pair ? pair_grid(p, units, x.device().index()) : tile_grid(p, tiles, x.device().index());
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_swiglu(p, dim3(grid, 1), BN, static_cast<int>(passes), stream, pair);
}
}  // namespace

// SwiGLU backward through the hidden layer: dh = dy @ w_down^T, then
// dgu[:, :Mh] = dh * u * silu'(g), dgu[:, Mh:] = dh * silu(g).
void gemm_swiglu_bwd(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u, torch::Tensor dgu,
                     int64_t passes) {
  gemm_swiglu_bwd_impl(dy, w_down, g, u, dgu, passes, Comm{});
}

void gemm_swiglu_bwd_tp(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u, torch::Tensor dgu,
                        int64_t passes, std::vector<int64_t> wait) {
  gemm_swiglu_bwd_impl(dy, w_down, g, u, dgu, passes, make_comm(wait, c10::nullopt));
}

namespace {
void gemm_swiglu_bwd_impl(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u, torch::Tensor dgu,
                          int64_t passes, const Comm& cm) {
  check_passes(passes);
  const c10::cuda::CUDAGuard guard(dy.device());
  Operand A = operand_of(dy, false, "dy");
  // w_down is (Mh, D): as B (K = D, N = Mh) it is stored [N][K], i.e. K-major.
  Operand B = operand_of(w_down, false, "w_down");
  TORCH_CHECK(B.k == A.k, "w_down shape");
  const int64_t T = A.mn, Mh = B.mn;
  TORCH_CHECK(g.size(0) == T && g.size(1) == Mh && u.sizes() == g.sizes() && u.stride(0) == g.stride(0), "g/u shape");
  TORCH_CHECK(dgu.size(0) == T && dgu.size(1) == 2 * Mh, "dgu must be (T, 2*hidden)");
  if (T == 0 || Mh == 0) return;
  const int BN = passes == 3 ? 128 : (Mh >= 2048 ? 256 : 128);
  const bool pair = use_pair(passes, T, !cm.wait.empty());
  Params p;
  memset(&p, 0, sizeof(p));
  p.tma_a = map_for(A, BM);
  p.tma_b[0] = map_for(B, pair ? BN / 2 : BN);
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(Mh);
  p.K = static_cast<int>(A.k);
  p.b_mode = kBSingle;
  p.num_n_tiles = static_cast<int>((Mh + BN - 1) / BN);
  p.alpha = 1.f;
  p.g_in = g.data_ptr<float>();
  p.u_in = u.data_ptr<float>();
  p.ld_gu = g.stride(0);
  p.dgu = dgu.data_ptr<float>();
  p.ld_dgu = dgu.stride(0);
  p.status = host::status_ptr(dy.device().index());
  apply_comm(p, cm, false, false);
  p.k_tiles_per_split = static_cast<int>((A.k + BK - 1) / BK);
  const long long tiles = ((T + BM - 1) / BM) * p.num_n_tiles;
  const long long units = ((T + 2 * BM - 1) / (2 * BM)) * p.num_n_tiles;
  p.splits = 1;
  p.batch_z = 1;
  const unsigned grid = pair ? pair_grid(p, units, dy.device().index()) : tile_grid(p, tiles, dy.device().index());
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_swiglu_bwd(p, dim3(grid, 1), BN, static_cast<int>(passes), stream, pair);
}
}  // namespace

}  // namespace gemm
}  // namespace abacus

