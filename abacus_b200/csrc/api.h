// Declarations of every op exported by the abacus_b200._C extension.
#pragma once
#include <torch/extension.h>
#include <vector>

namespace abacus {
namespace gemm {
void gemm_out(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
              int64_t b_mode, double alpha, c10::optional<torch::Tensor> residual, bool accumulate, int64_t passes);
int64_t gemm_n_tiles(int64_t n, int64_t passes);
int64_t gemm_pair_clusters();
void gemm_qkv_norm_rope(torch::Tensor qkv, torch::Tensor x, std::vector<torch::Tensor> ws, torch::Tensor q,
                        torch::Tensor k, torch::Tensor rstd, torch::Tensor q_gamma, torch::Tensor k_gamma,
                        torch::Tensor cos_t, torch::Tensor sin_t, int64_t seq_len, int64_t heads, int64_t head_dim,
                        double eps, int64_t passes);
void gemm_trace(c10::optional<torch::Tensor> buf);
int64_t gemm_grouped(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
                     int64_t b_mode, double alpha, bool accumulate, int64_t passes,
                     c10::optional<std::vector<int64_t>> scatter);
void gemm_swiglu_grouped(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                         torch::Tensor h, int64_t passes, c10::optional<std::vector<int64_t>> wait);
void gemm_swiglu_bwd_grouped(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u,
                             torch::Tensor dgu, int64_t passes, c10::optional<std::vector<int64_t>> wait);
int64_t gemm_out_tp(torch::Tensor c, torch::Tensor a, std::vector<torch::Tensor> bs, bool trans_a, bool trans_b,
                    int64_t b_mode, double alpha, int64_t passes, c10::optional<std::vector<int64_t>> wait,
                    c10::optional<std::vector<int64_t>> scatter);
void gemm_swiglu_tp(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                    torch::Tensor h, int64_t passes, std::vector<int64_t> wait);
void gemm_swiglu_bwd_tp(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u, torch::Tensor dgu,
                        int64_t passes, std::vector<int64_t> wait);
void gemm_batched(torch::Tensor c, torch::Tensor a, torch::Tensor b, bool trans_a, bool trans_b, double alpha,
                  int64_t causal, int64_t passes);
void gemm_swiglu(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up, torch::Tensor g, torch::Tensor u,
                 torch::Tensor h, int64_t passes);
void gemm_swiglu_bwd(torch::Tensor dy, torch::Tensor w_down, torch::Tensor g, torch::Tensor u, torch::Tensor dgu,
                     int64_t passes);
}  // namespace gemm
}  // namespace abacus

namespace abacus {
namespace ops {
void rmsnorm_fwd(torch::Tensor x, torch::Tensor gamma, torch::Tensor y, torch::Tensor rstd, double eps);
void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor gamma, torch::Tensor rstd, torch::Tensor dx,
                 torch::Tensor dgamma);
void qk_prologue_fwd(torch::Tensor qkv, torch::Tensor gq, torch::Tensor gk, torch::Tensor cos_t, torch::Tensor sin_t,
                     c10::optional<torch::Tensor> positions, int64_t seq_len, torch::Tensor q_out, torch::Tensor k_out,
                     torch::Tensor rstd, int64_t heads, int64_t head_dim, double eps);
void qk_prologue_bwd(torch::Tensor qkv, torch::Tensor gq, torch::Tensor gk, torch::Tensor cos_t, torch::Tensor sin_t,
                     c10::optional<torch::Tensor> positions, int64_t seq_len, torch::Tensor dq, torch::Tensor dk,
                     torch::Tensor rstd, torch::Tensor dqkv, torch::Tensor dgq, torch::Tensor dgk, int64_t heads,
                     int64_t head_dim);
void embedding_fwd(torch::Tensor tokens, torch::Tensor weight, torch::Tensor out);
void embedding_bwd(torch::Tensor sorted_tokens, torch::Tensor perm, torch::Tensor dy, torch::Tensor dw);
void cross_entropy_fwd_bwd(torch::Tensor logits, torch::Tensor target, torch::Tensor loss, c10::optional<torch::Tensor> lse,
                           int64_t ignore_index, torch::Tensor grad_scale, bool write_grad);
void cross_entropy_grad(torch::Tensor logits, torch::Tensor grad, torch::Tensor target, torch::Tensor lse,
                        int64_t ignore_index, torch::Tensor grad_scale);
void adamw_step(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads, std::vector<torch::Tensor> exp_avgs,
                std::vector<torch::Tensor> exp_avg_sqs, double lr, double beta1, double beta2, double eps,
                double weight_decay, int64_t step);
}  // namespace ops
}  // namespace abacus

namespace abacus {
namespace attn {
void causal_softmax_fwd(torch::Tensor s);
void causal_softmax_bwd(torch::Tensor p, torch::Tensor dp, double scale);
void flash_attn_fwd_cp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       int64_t batch, int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                       c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                       std::vector<int64_t> wait);
void flash_attn_bwd_cp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
                       torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, int64_t batch,
                       int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                       c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                       std::vector<int64_t> scatter);
void flash_fwd_trace(c10::optional<torch::Tensor> buf);
void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    int64_t batch, int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes);
void flash_attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, int64_t batch,
                    int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes);
}  // namespace attn
}  // namespace abacus

namespace abacus {
namespace comm {
void wait_flag(torch::Tensor flag, int64_t expected, double timeout_ms, torch::Tensor result);
void set_flag(torch::Tensor flag, int64_t value);
void symm_barrier(std::vector<int64_t> signal_ptrs, int64_t rank, int64_t slot_base, int64_t epoch, double timeout_ms,
                  std::vector<int64_t> exch_ptrs, c10::optional<torch::Tensor> payload);
void tp_push_rows(torch::Tensor x, std::vector<int64_t> dst_ptrs, std::vector<int64_t> flag_ptrs, int64_t chunk,
                  int64_t seq, int64_t self, int64_t epoch, torch::Tensor done);
void tp_reduce_rows(torch::Tensor staging, int64_t world, torch::Tensor counters, int64_t target,
                    c10::optional<torch::Tensor> residual, torch::Tensor out);
void ep_push_rows(torch::Tensor src, int64_t top_k, torch::Tensor dest_rank, torch::Tensor dest_row,
                  c10::optional<torch::Tensor> scale, std::vector<int64_t> row_ptrs, std::vector<int64_t> meta_ptrs,
                  std::vector<int64_t> flag_ptrs, int64_t self, int64_t epoch, torch::Tensor done);
void ep_credit(torch::Tensor counter, torch::Tensor amount, int64_t multiplier);
void ep_combine(torch::Tensor ret, c10::optional<torch::Tensor> weights, int64_t top_k, torch::Tensor counter,
                int64_t target, torch::Tensor out);
void ar_adamw(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs, torch::Tensor counts, bool normalize,
              int64_t rank, int64_t lo, int64_t hi, torch::Tensor exp_avg, torch::Tensor exp_avg_sq, double lr,
              double beta1, double beta2, double eps, double weight_decay, int64_t step, int64_t max_ctas,
              c10::optional<torch::Tensor> local_param);
}  // namespace comm
}  // namespace abacus
