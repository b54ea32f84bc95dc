// Raw-pointer launch API of the CUDA kernels (no torch types); bindings.cpp validates tensors and calls these.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace qw {

using bf16 = __nv_bfloat16;

inline void check_cuda(cudaError_t err, const char* what) {
  if (err != cudaSuccess) throw std::runtime_error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(err));
}

// ---- gemm.cu (tcgen05) ----
void linear_fwd(const bf16* x, int64_t ldx, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                const float* bias, const bf16* residual, int64_t ldr, void* out, int64_t ldo, bool out_fp32,
                cudaStream_t stream);
void linear_dgrad(const bf16* dy, int64_t lddy, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K, void* dx,
                  int64_t lddx, bool out_fp32, bool accumulate, cudaStream_t stream);
void linear_wgrad(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, int64_t T, int64_t N, int64_t K, void* dw,
                  int64_t lddw, bool out_fp32, bool accumulate, cudaStream_t stream);
// Grouped MoE GEMMs. `G` groups of rows (counts/offsets), group g uses expert weight block g % E (E = weight
// stack size; G = sources * E for expert-parallel receive buffers).
void moe_gate_up_fwd(const bf16* x, const bf16* w_gate_up, const int* counts, const int* offsets, int64_t R, int64_t G,
                     int64_t E, int64_t H, int64_t F, bf16* h, bf16* gu, cudaStream_t stream);
void moe_down_fwd(const bf16* h, const bf16* w_down, const int* counts, const int* offsets, int64_t R, int64_t G,
                  int64_t E, int64_t H, int64_t F, bf16* y, cudaStream_t stream, void* const* peer_out = nullptr,
                  int64_t peer_rows = 0, int peer_slot = 0);
void moe_down_bwd(const bf16* dy, const bf16* w_down, const int* counts, const int* offsets, int64_t R, int64_t G,
                  int64_t E, int64_t H, int64_t F, const bf16* gu, const float* route_w, bf16* dgu, bf16* h_weighted,
                  float* dw_partial, int dw_tiles, cudaStream_t stream);
int moe_dw_tiles(int64_t F);
void moe_gate_up_dgrad(const bf16* dgu, const bf16* w_gate_up, const int* counts, const int* offsets, int64_t R,
                       int64_t G, int64_t E, int64_t H, int64_t F, bf16* dx, cudaStream_t stream, void* const* peer_out = nullptr,
                       int64_t peer_rows = 0, int peer_slot = 0);
// out[e] (+)= sum over the `segments` row groups s*E + e of a^T b   (segments = sources in expert parallelism)
void moe_wgrad(const bf16* a, const bf16* b, const int* counts, const int* offsets, int64_t R, int64_t E, int segments,
               int64_t M, int64_t N, void* out, bool out_fp32, bool accumulate, float alpha, cudaStream_t stream);
int gemm_status(bool clear);
void gemm_trace(void* buf);
void attn_fwd_trace(void* buf);
void attn_bwd_trace(void* buf);  // timeline of the backward's CTA (0, 0) (null disarms)  // timeline of the forward's CTA (0, 0) (null disarms)  // per-tile clock64 timestamps of CTA 0 (null disarms)
int wgrad_split(int64_t T, int64_t N, int64_t K);
void splitk_reduce(const float* partial, int chunks, int64_t rows, int64_t cols, void* out, int64_t ldo,
                   bool out_fp32, bool accumulate, cudaStream_t stream);

// ---- norm_rope.cu ----
void norm_fwd(const bf16* x, const bf16* delta, bf16* x_out, const float* w, const float* b, bf16* y, float* mean,
              float* rstd, int64_t rows, int H, float eps, bool rms, cudaStream_t stream);
int norm_bwd_blocks(int64_t rows);
int bias_grad_slabs(int64_t rows);
void bias_grad(const bf16* g, int64_t ldg, int64_t rows, int N, float* part, float* out, bool accumulate,
               cudaStream_t stream);
void norm_bwd(const bf16* dy, const bf16* x, const float* w, const float* mean, const float* rstd, const bf16* dres,
              bf16* dx, float* dw_part, float* db_part, float* dw, float* db, int64_t rows, int H, bool rms,
              bool accumulate, cudaStream_t stream);
void rope_apply(bf16* qkv, int64_t rows, int heads_rot, int D, int64_t ld, int seq, const int* positions,
                const float* cos_t, const float* sin_t, bool inverse, cudaStream_t stream);
int norm_status(bool clear);

// ---- moe_routing.cu ----
void router_logits(const bf16* x, const float* w, int64_t T, int H, int E, float* logits, cudaStream_t stream);
void router_topk(const float* logits, const float* bias, int64_t T, int E, int k, float temperature, float* probs,
                 int* top_idx, float* top_w, int* counts, cudaStream_t stream);
int moe_plan_chunks(int64_t routes);
void moe_plan(const int* top_idx, const float* top_w, const int* counts, int64_t routes, int E, int cap, int slot_rows,
              int* kept, int* offsets, int* uoffsets, int* meta, int* chunk_hist, int* sorted_routes, int* route_row,
              cudaStream_t stream);
void moe_permute(const bf16* x, int64_t routes, int k, int H, const int* route_row, const float* top_w, const int* kept,
                 const int* offsets, int E, bf16* x_perm, int* row_token, float* row_w, int64_t perm_rows,
                 cudaStream_t stream);
void moe_pad_zero(const int* kept, const int* offsets, int E, int H, bf16* buf, cudaStream_t stream);
void moe_gather_rows(const bf16* src, const int* row_token, const int* meta, int64_t max_rows, int H, bf16* dst,
                     cudaStream_t stream);
void moe_combine(const bf16* y, const int* route_row, const float* top_w, const bf16* resid, int64_t T, int k, int H,
                 bf16* out, int64_t y_rows, cudaStream_t stream);
void moe_combine_grad(const bf16* dx_perm, const int* route_row, const float* extra, int64_t T, int k, int H, bf16* dx,
                      int64_t perm_rows, cudaStream_t stream);
void moe_route_dw(const float* partial, int tiles, const int* route_row, int64_t routes, float* d_w,
                  cudaStream_t stream);
void router_backward(const float* probs, const int* top_idx, const float* top_w, const float* d_w,
                     const float* d_probs_ext, int64_t T, int E, int k, float temperature, float* d_logits,
                     cudaStream_t stream);
void router_dx(const float* d_logits, const float* w, int64_t T, int E, int H, float* dx, cudaStream_t stream);
int router_dw_split(int64_t T);
// tensor-core router GEMMs (fp32 operands split into bf16 parts); scratch: w3 [3E,H] bf16, out3 [T,3E] fp32,
// dls [T,3E] bf16, partial [ceil(T/router_dw_chunk) * 2E * H] fp32
bool router_tc_ok(int64_t T, int H, int E);
void router_logits_tc(const bf16* x, const float* w, int64_t T, int H, int E, float* logits, bf16* w3, float* out3,
                      cudaStream_t stream);
void router_dx_tc(const float* d_logits, const float* w, int64_t T, int E, int H, float* dx, bf16* dls, bf16* w3,
                  cudaStream_t stream);
int64_t router_dw_chunk(int64_t T, int H);
void router_dw_tc(const float* d_logits, const bf16* x, int64_t T, int E, int H, float* dw, bool accumulate,
                  bf16* dls, float* partial, cudaStream_t stream);
// fused tensor parallelism: GEMMs whose epilogue stores rows into peers' staging buffers, and the reduction that
// sums the staged partials and stores the result into every rank's output buffer (tp_fused.cu)
void linear_fwd_peer(const bf16* x, int64_t ldx, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                     void* const* peer_out, int64_t peer_rows, int peer_slot, cudaStream_t stream);
void linear_dgrad_peer(const bf16* dy, int64_t lddy, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                       void* const* peer_out, int64_t peer_rows, int peer_slot, cudaStream_t stream);
void tp_reduce_rows(const bf16* staging, int world, int64_t rows_per_rank, int N, const float* bias, bf16* out,
                    cudaStream_t stream);
void tp_reduce_bcast(const bf16* staging, int world, int64_t rows_per_rank, int N, const float* bias,
                     void* const* outs, int me, cudaStream_t stream);
int tp_status(bool clear);
void linear_wgrad_chunks(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, int64_t T, int64_t N, int64_t K,
                         int64_t chunk, float* partial, cudaStream_t stream);
void router_dw(const float* d_logits, const bf16* x, int64_t T, int E, int H, float* dw, bool accumulate,
               float* workspace, cudaStream_t stream);
int routing_status(bool clear);

// ---- optim_ce.cu ----
struct AdamTensor {
  void* param;         // bf16 (with master) or fp32 (updated in place)
  const void* grad;    // fp32 (grad_dtype 0) or bf16 (grad_dtype 1)
  float* master;       // fp32 master copy, or nullptr when the parameter itself is fp32
  float* exp_avg;
  float* exp_avg_sq;
  int64_t numel;
  int grad_dtype;
  float decay_scale;   // 1 = apply weight decay, 0 = exempt
  float grad_scale;    // multiplies the stored gradient (e.g. 1/ep for expert gradients summed over ranks)
  int reserved;        // keeps the record at 64 bytes (mirrored by the Python table builder)
};
struct AdamHyper {
  float lr, beta1, beta2, eps, weight_decay, bias_correction1, bias_correction2_sqrt;
};
int adam_chunk_size();
void adam_grad_norm(const AdamTensor* tensors, const int* chunk_tensor, const int64_t* chunk_start, int chunks,
                    double* partial, const double* extra_sumsq, float max_norm, float* norm_out, cudaStream_t stream);
void adam_sumsq(const AdamTensor* tensors, const int* chunk_tensor, const int64_t* chunk_start, int chunks,
                double* partial, cudaStream_t stream);
// small_blocks > 0: 128-thread blocks, at most small_blocks of them striding over the chunks (an update that runs
// beside other kernels)
void adam_step(const AdamTensor* tensors, const int* chunk_tensor, const int64_t* chunk_start, int chunks,
               const AdamHyper& hyper, const float* clip, bool eight_bit, cudaStream_t stream, int small_blocks = 0);
int adam8_block_size();
void cross_entropy_chunk(bf16* logits, int64_t rows, int64_t ld, int V, const int64_t* labels, float grad_scale,
                         float* loss_out, int ignore_index, cudaStream_t stream);
void scale_bf16(bf16* x, int64_t n, const float* scale, cudaStream_t stream);
int optim_status(bool clear);

// ---- attention.cu ----
void flash_attn_fwd(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, bf16* o,
                    int64_t ldo, float* lse, int B, int S, int Hq, int Hkv, int D, float scale, cudaStream_t stream);
void flash_attn_bwd(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, const bf16* o,
                    int64_t ldo, const bf16* dout, int64_t lddo, const float* lse, float* delta, bf16* dq,
                    int64_t lddq, bf16* dk, int64_t lddk, bf16* dv, int64_t lddv, int B, int S, int Hq, int Hkv, int D,
                    float scale, cudaStream_t stream);
int attention_status(bool clear);
// tcgen05 backward (dK/dV and dQ kernels) for head_dim 64 / 128; `delta` must already hold rowsum(dO * O)
void flash_attn_bwd_tc(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv,
                       const bf16* dout, int64_t lddo, const float* lse, const float* delta, bf16* dq, int64_t lddq,
                       bf16* dk, int64_t lddk, bf16* dv, int64_t lddv, int B, int S, int Hq, int Hkv, int D,
                       float scale, cudaStream_t stream);
int attention_tc_status(bool clear);
// tcgen05 causal flash-attention forward, head_dim 64 (attention_fwd_tc.cu)
void flash_attn_fwd_tc(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, bf16* o,
                       int64_t ldo, float* lse, int B, int S, int Hq, int Hkv, int D, float scale,
                       cudaStream_t stream);
int attention_fwd_tc_status(bool clear);
int ep_status(bool clear);

// ---- p2p.cu ----
void p2p_broadcast(const void* src, int64_t block_bytes, void* const* peer_bufs, int* const* peer_flags, int world,
                   int me, int epoch, unsigned int* done, cudaStream_t stream);
void p2p_push(const void* src, int64_t block_bytes, void* const* peer_bufs, int* const* peer_flags, int world, int me,
              int epoch, unsigned int* done, cudaStream_t stream);
void p2p_wait(const int* flags, int world, int epoch, double timeout_s, cudaStream_t stream);
int p2p_status(bool clear);

// ---- ep_fused.cu (expert-parallel dispatch / return over peer memory) ----
void ep_dispatch(const bf16* x, int64_t T, int k, int H, const int* route_row, const float* top_w, const int* kept,
                 int E, int local, int slot, int me, int world, uint8_t* const* peer, int64_t w_off, int64_t c_off,
                 int* const* peer_flags, int epoch, unsigned int* done, cudaStream_t stream);
void ep_pad(const int* counts, int groups, int slot, int H, bf16* rows, float* w, cudaStream_t stream);
void ep_signal(int* const* peer_flags, int world, int me, int epoch, cudaStream_t stream);
// ---- zero_fused.cu (ZeRO reduce-scatter and AdamW + all-gather over peer memory) ----
int zero_rs_blocks(int64_t per);
void zero_reduce_scatter(const void* const* peers, int world, int dtype, int64_t start, int64_t per, float* shard,
                         double* partial, cudaStream_t stream);
void zero_adamw_gather(float* master, float* m, float* v, const float* grad, const float* clip, const AdamHyper& h,
                       void* const* peers, int world, int dtype, int64_t start, int64_t per, int64_t valid,
                       cudaStream_t stream);

// ---- decode.cu ----
void grouped_gemv(const bf16* x, int64_t ldx, const void* w, const void* scales, int64_t w_group_bytes,
                  int64_t s_group_elems, int N, int K, int group, int fmt, bool swiglu, const int* tok, const int* off,
                  const int* cnt, int groups, int dense_rows, bf16* out, int64_t ldo, bool out_by_route,
                  const float* bias, const bf16* resid, int64_t ldr, const int* active, int active_slots,
                  cudaStream_t stream);
int decode_attn_chunks(int Lmax);
// first/local: the experts this rank holds (expert-parallel decode); `active` lists them relative to `first`
void decode_route(const bf16* x, const float* wr, const float* ebias, int T, int H, int E, int k, float temperature,
                  float* logits, int* cnt, int* off, int* order, int* route_slot, float* top_w, int* active,
                  int* ticket, cudaStream_t stream, int first = 0, int local = -1);
void decode_attention(const bf16* q, const bf16* kc, const bf16* vc, const int* lens, int B, int Hq, int Hkv, int D,
                      int Lmax, float scale, float* part_o, float* part_ml, int* tickets, bf16* out,
                      cudaStream_t stream);
// decode attention from the raw QKV row with RoPE and the KV-cache append of the new token (pos[b]) folded in
void decode_attention_rope(const bf16* qkv, const int* pos, const float* cos_t, const float* sin_t, bool rope,
                           bf16* kc, bf16* vc, int B, int Hq, int Hkv, int D, int Lmax, float scale, float* part_o,
                           float* part_ml, int* tickets, bf16* out, cudaStream_t stream);
void rope_append(const bf16* qkv, const int* pos, int B, int Hq, int Hkv, int D, int Lmax, const float* cos_t,
                 const float* sin_t, bool rope, bf16* q_out, bf16* kc, bf16* vc, cudaStream_t stream);
// parts: expert-parallel partial MoE outputs (ep_decode.cu planes) summed in rank order instead of y/slot/top_w
void decode_combine_norm(const bf16* x, const int64_t* tokens, const bf16* tok_emb, const bf16* pos_emb,
                         const int* positions, const bf16* y, const int* slot, const float* top_w, int k, int T, int H,
                         const float* w, const float* bias, float eps, bool rms, bf16* x_out, bf16* n_out,
                         cudaStream_t stream, const float* parts = nullptr, const int* part_step = nullptr,
                         int part_layer = 0, int part_layers = 1, int part_world = 1, int part_tstride = 0);
int decode_status(bool clear);
// bf16 copy of int4 (fmt 2, grouped fp16 scales) / int8 (fmt 1, per-row fp16 scale) weight rows
void dequant_rows(const void* q, const void* scales, int64_t rows, int K, int group, int fmt, bf16* out,
                  cudaStream_t stream);
// expert-parallel decode exchange (ep_decode.cu)
void ep_decode_tick(int* step, cudaStream_t stream);
void ep_decode_push(const bf16* y, const int* slot, const float* top_w, int k, int T, int H, int tstride,
                    float* const* peers, int64_t plane_floats, int layer, int layers, int me, int world,
                    int* const* peer_flags, const int* step, unsigned int* done, cudaStream_t stream);
void ep_decode_wait(const int* flags, int world, const int* step, int layer, int layers, double timeout_s,
                    cudaStream_t stream);
int ep_decode_status(bool clear);

}  // namespace qw
