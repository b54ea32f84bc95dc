// PyTorch bindings: tensor validation and stream selection around the raw-pointer launchers (launchers.h).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "launchers.h"

namespace {

using torch::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_DTYPE(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has the wrong dtype")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_ROWS(t) TORCH_CHECK((t).dim() == 2 && (t).stride(1) == 1, #t " must be 2-D with unit inner stride")

const qw::bf16* bptr(const Tensor& t) { return reinterpret_cast<const qw::bf16*>(t.data_ptr()); }
qw::bf16* bptr_mut(const Tensor& t) { return reinterpret_cast<qw::bf16*>(t.data_ptr()); }
template <typename T>
const T* optptr(const OptT& t) { return t && t->defined() ? t->data_ptr<T>() : nullptr; }
const qw::bf16* optb(const OptT& t) { return t && t->defined() ? bptr(*t) : nullptr; }
qw::bf16* optb_mut(const OptT& t) { return t && t->defined() ? bptr_mut(*t) : nullptr; }

// ------------------------------------------------------------------------------------------------ GEMM
void linear_fwd(Tensor x, Tensor w, OptT bias, OptT residual, Tensor out) {
  CHECK_CUDA(x); CHECK_ROWS(x); CHECK_DTYPE(x, torch::kBFloat16);
  CHECK_ROWS(w); CHECK_DTYPE(w, torch::kBFloat16); CHECK_ROWS(out);
  TORCH_CHECK(w.size(1) == x.size(1) && out.size(0) == x.size(0) && out.size(1) == w.size(0), "linear_fwd shapes");
  if (bias) { CHECK_DTYPE(*bias, torch::kFloat32); TORCH_CHECK(bias->numel() == w.size(0)); }
  if (residual) { CHECK_ROWS(*residual); CHECK_DTYPE(*residual, torch::kBFloat16); }
  const bool fp32 = out.scalar_type() == torch::kFloat32;
  TORCH_CHECK(fp32 || out.scalar_type() == torch::kBFloat16);
  c10::cuda::CUDAGuard g(x.device());
  qw::linear_fwd(bptr(x), x.stride(0), bptr(w), w.stride(0), x.size(0), w.size(0), x.size(1), optptr<float>(bias),
                 optb(residual), residual ? residual->stride(0) : 0, out.data_ptr(), out.stride(0), fp32, stream());
}

void linear_dgrad(Tensor dy, Tensor w, Tensor dx, bool accumulate) {
  CHECK_CUDA(dy); CHECK_ROWS(dy); CHECK_DTYPE(dy, torch::kBFloat16);
  CHECK_ROWS(w); CHECK_DTYPE(w, torch::kBFloat16); CHECK_ROWS(dx);
  TORCH_CHECK(w.size(0) == dy.size(1) && dx.size(0) == dy.size(0) && dx.size(1) == w.size(1), "linear_dgrad shapes");
  const bool fp32 = dx.scalar_type() == torch::kFloat32;
  c10::cuda::CUDAGuard g(dy.device());
  qw::linear_dgrad(bptr(dy), dy.stride(0), bptr(w), w.stride(0), dy.size(0), dy.size(1), w.size(1), dx.data_ptr(),
                   dx.stride(0), fp32, accumulate, stream());
}

// tensor-parallel partial products into the owners' staging buffers (peer pointers: int64 device tensor [world])
void linear_fwd_peer(Tensor x, Tensor w, Tensor peer_ptrs, int64_t peer_rows, int64_t slot) {
  CHECK_CUDA(x); CHECK_ROWS(x); CHECK_DTYPE(x, torch::kBFloat16);
  CHECK_ROWS(w); CHECK_DTYPE(w, torch::kBFloat16); CHECK_DTYPE(peer_ptrs, torch::kInt64);
  TORCH_CHECK(w.size(1) == x.size(1) && x.size(0) % peer_rows == 0, "linear_fwd_peer shapes");
  c10::cuda::CUDAGuard g(x.device());
  qw::linear_fwd_peer(bptr(x), x.stride(0), bptr(w), w.stride(0), x.size(0), w.size(0), x.size(1),
                      reinterpret_cast<void* const*>(peer_ptrs.data_ptr<int64_t>()), peer_rows, static_cast<int>(slot),
                      stream());
}

void linear_dgrad_peer(Tensor dy, Tensor w, Tensor peer_ptrs, int64_t peer_rows, int64_t slot) {
  CHECK_CUDA(dy); CHECK_ROWS(dy); CHECK_DTYPE(dy, torch::kBFloat16);
  CHECK_ROWS(w); CHECK_DTYPE(w, torch::kBFloat16); CHECK_DTYPE(peer_ptrs, torch::kInt64);
  TORCH_CHECK(w.size(0) == dy.size(1) && dy.size(0) % peer_rows == 0, "linear_dgrad_peer shapes");
  c10::cuda::CUDAGuard g(dy.device());
  qw::linear_dgrad_peer(bptr(dy), dy.stride(0), bptr(w), w.stride(0), dy.size(0), dy.size(1), w.size(1),
                        reinterpret_cast<void* const*>(peer_ptrs.data_ptr<int64_t>()), peer_rows,
                        static_cast<int>(slot), stream());
}

void tp_reduce_rows(Tensor staging, int64_t world, int64_t rows_per_rank, int64_t N, OptT bias, Tensor out) {
  CHECK_CUDA(staging); CHECK_DTYPE(staging, torch::kBFloat16); CHECK_DTYPE(out, torch::kBFloat16); CHECK_CONTIG(out);
  TORCH_CHECK(out.numel() == rows_per_rank * N, "tp_reduce_rows: output size");
  if (bias) { CHECK_DTYPE(*bias, torch::kFloat32); TORCH_CHECK(bias->numel() == N); }
  c10::cuda::CUDAGuard g(staging.device());
  qw::tp_reduce_rows(bptr(staging), static_cast<int>(world), rows_per_rank, static_cast<int>(N), optptr<float>(bias),
                     bptr_mut(out), stream());
}

void tp_reduce_bcast(Tensor staging, int64_t world, int64_t rows_per_rank, int64_t N, OptT bias, Tensor out_ptrs,
                     int64_t me) {
  CHECK_CUDA(staging); CHECK_DTYPE(staging, torch::kBFloat16); CHECK_DTYPE(out_ptrs, torch::kInt64);
  if (bias) { CHECK_DTYPE(*bias, torch::kFloat32); TORCH_CHECK(bias->numel() == N); }
  c10::cuda::CUDAGuard g(staging.device());
  qw::tp_reduce_bcast(bptr(staging), static_cast<int>(world), rows_per_rank, static_cast<int>(N), optptr<float>(bias),
                      reinterpret_cast<void* const*>(out_ptrs.data_ptr<int64_t>()), static_cast<int>(me), stream());
}

void linear_wgrad(Tensor dy, Tensor x, Tensor dw, bool accumulate) {
  CHECK_CUDA(dy); CHECK_ROWS(dy); CHECK_DTYPE(dy, torch::kBFloat16);
  CHECK_ROWS(x); CHECK_DTYPE(x, torch::kBFloat16); CHECK_ROWS(dw);
  TORCH_CHECK(x.size(0) == dy.size(0) && dw.size(0) == dy.size(1) && dw.size(1) == x.size(1), "linear_wgrad shapes");
  const bool fp32 = dw.scalar_type() == torch::kFloat32;
  c10::cuda::CUDAGuard g(dy.device());
  const int64_t T = dy.size(0), N = dy.size(1), K = x.size(1);
  const int split = qw::wgrad_split(T, N, K);
  if (split > 1) {  // too few output tiles to fill the GPU: split the token reduction, then a fixed-order sum
    const int64_t chunk = ((T + split - 1) / split + 63) / 64 * 64;
    const int chunks = static_cast<int>((T + chunk - 1) / chunk);
    auto partial = torch::empty({chunks, N, K}, dy.options().dtype(torch::kFloat32));
    qw::linear_wgrad_chunks(bptr(dy), dy.stride(0), bptr(x), x.stride(0), T, N, K, chunk, partial.data_ptr<float>(),
                            stream());
    qw::splitk_reduce(partial.data_ptr<float>(), chunks, N, K, dw.data_ptr(), dw.stride(0), fp32, accumulate,
                      stream());
    return;
  }
  qw::linear_wgrad(bptr(dy), dy.stride(0), bptr(x), x.stride(0), T, N, K, dw.data_ptr(), dw.stride(0), fp32,
                   accumulate, stream());
}

void check_groups(const Tensor& counts, const Tensor& offsets, int64_t E) {
  CHECK_DTYPE(counts, torch::kInt32); CHECK_DTYPE(offsets, torch::kInt32);
  TORCH_CHECK(counts.numel() >= E && offsets.numel() >= E, "group tables too short");
}

void moe_gate_up_fwd(Tensor x, Tensor w, Tensor counts, Tensor offsets, Tensor h, OptT gu) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_CONTIG(w); CHECK_CONTIG(h); CHECK_DTYPE(w, torch::kBFloat16);
  const int64_t E = w.size(0), F = w.size(1) / 2, H = w.size(2), R = x.size(0);
  TORCH_CHECK(x.size(1) == H && h.size(0) == R && h.size(1) == F, "moe_gate_up_fwd shapes");
  if (gu) { CHECK_CONTIG(*gu); TORCH_CHECK(gu->size(0) == R && gu->size(1) == 2 * F); }
  const int64_t G = counts.numel();
  check_groups(counts, offsets, G);
  TORCH_CHECK(G % E == 0, "groups must be a multiple of the expert count");
  c10::cuda::CUDAGuard g(x.device());
  qw::moe_gate_up_fwd(bptr(x), bptr(w), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, G, E, H, F, bptr_mut(h),
                      optb_mut(gu), stream());
}

void moe_down_fwd(Tensor h, Tensor w, Tensor counts, Tensor offsets, Tensor y) {
  CHECK_CUDA(h); CHECK_CONTIG(h); CHECK_CONTIG(w); CHECK_CONTIG(y);
  const int64_t E = w.size(0), H = w.size(1), F = w.size(2), R = h.size(0);
  TORCH_CHECK(h.size(1) == F && y.size(0) == R && y.size(1) == H, "moe_down_fwd shapes");
  const int64_t G = counts.numel();
  check_groups(counts, offsets, G);
  TORCH_CHECK(G % E == 0, "groups must be a multiple of the expert count");
  c10::cuda::CUDAGuard g(h.device());
  qw::moe_down_fwd(bptr(h), bptr(w), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, G, E, H, F, bptr_mut(y),
                   stream());
}

// peer_ptrs: int64 [world] base address of every rank's receive buffer (bf16 [world * peer_rows, H]); row r of the
// result goes to rank r / peer_rows at row peer_slot * peer_rows + r % peer_rows
static void* const* peer_table(const Tensor& peer_ptrs, int64_t peer_rows, int64_t R) {
  CHECK_CUDA(peer_ptrs);
  CHECK_DTYPE(peer_ptrs, torch::kInt64);
  TORCH_CHECK(peer_rows > 0 && R == peer_ptrs.numel() * peer_rows, "peer table: rows must be world * peer_rows");
  return reinterpret_cast<void* const*>(peer_ptrs.data_ptr<int64_t>());
}

void moe_down_fwd_peer(Tensor h, Tensor w, Tensor counts, Tensor offsets, Tensor peer_ptrs, int64_t peer_rows,
                       int64_t peer_slot) {
  CHECK_CUDA(h); CHECK_CONTIG(h); CHECK_CONTIG(w);
  const int64_t E = w.size(0), H = w.size(1), F = w.size(2), R = h.size(0);
  TORCH_CHECK(h.size(1) == F, "moe_down_fwd_peer shapes");
  const int64_t G = counts.numel();
  check_groups(counts, offsets, G);
  TORCH_CHECK(G % E == 0, "groups must be a multiple of the expert count");
  TORCH_CHECK(peer_slot >= 0 && peer_slot < peer_ptrs.numel(), "peer slot out of range");
  c10::cuda::CUDAGuard g(h.device());
  qw::moe_down_fwd(bptr(h), bptr(w), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, G, E, H, F, nullptr,
                   stream(), peer_table(peer_ptrs, peer_rows, R), peer_rows, static_cast<int>(peer_slot));
}

void moe_gate_up_dgrad_peer(Tensor dgu, Tensor w, Tensor counts, Tensor offsets, Tensor peer_ptrs, int64_t peer_rows,
                            int64_t peer_slot) {
  CHECK_CUDA(dgu); CHECK_CONTIG(dgu); CHECK_CONTIG(w);
  const int64_t E = w.size(0), F = w.size(1) / 2, H = w.size(2), R = dgu.size(0);
  TORCH_CHECK(dgu.size(1) == 2 * F, "moe_gate_up_dgrad_peer shapes");
  const int64_t G = counts.numel();
  check_groups(counts, offsets, G);
  TORCH_CHECK(G % E == 0, "groups must be a multiple of the expert count");
  TORCH_CHECK(peer_slot >= 0 && peer_slot < peer_ptrs.numel(), "peer slot out of range");
  c10::cuda::CUDAGuard g(dgu.device());
  qw::moe_gate_up_dgrad(bptr(dgu), bptr(w), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, G, E, H, F, nullptr,
                        stream(), peer_table(peer_ptrs, peer_rows, R), peer_rows, static_cast<int>(peer_slot));
}

void moe_down_bwd(Tensor dy, Tensor w, Tensor counts, Tensor offsets, Tensor gu, Tensor route_w, Tensor dgu,
                  OptT h_weighted, Tensor dw_partial) {
  CHECK_CUDA(dy); CHECK_CONTIG(dy); CHECK_CONTIG(w); CHECK_CONTIG(gu); CHECK_CONTIG(dgu); CHECK_CONTIG(dw_partial);
  const int64_t E = w.size(0), H = w.size(1), F = w.size(2), R = dy.size(0);
  TORCH_CHECK(dy.size(1) == H && gu.size(0) == R && gu.size(1) == 2 * F && dgu.sizes() == gu.sizes(),
              "moe_down_bwd shapes");
  CHECK_DTYPE(route_w, torch::kFloat32);
  CHECK_DTYPE(dw_partial, torch::kFloat32);
  TORCH_CHECK(dw_partial.size(0) == R && dw_partial.size(1) == qw::moe_dw_tiles(F));
  if (h_weighted) TORCH_CHECK(h_weighted->size(0) == R && h_weighted->size(1) == F);
  const int64_t G = counts.numel();
  check_groups(counts, offsets, G);
  TORCH_CHECK(G % E == 0, "groups must be a multiple of the expert count");
  c10::cuda::CUDAGuard g(dy.device());
  qw::moe_down_bwd(bptr(dy), bptr(w), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, G, E, H, F, bptr(gu),
                   route_w.data_ptr<float>(), bptr_mut(dgu), optb_mut(h_weighted), dw_partial.data_ptr<float>(),
                   static_cast<int>(dw_partial.size(1)), stream());
}

void moe_gate_up_dgrad(Tensor dgu, Tensor w, Tensor counts, Tensor offsets, Tensor dx) {
  CHECK_CUDA(dgu); CHECK_CONTIG(dgu); CHECK_CONTIG(w); CHECK_CONTIG(dx);
  const int64_t E = w.size(0), F = w.size(1) / 2, H = w.size(2), R = dgu.size(0);
  TORCH_CHECK(dgu.size(1) == 2 * F && dx.size(0) == R && dx.size(1) == H, "moe_gate_up_dgrad shapes");
  const int64_t G = counts.numel();
  check_groups(counts, offsets, G);
  TORCH_CHECK(G % E == 0, "groups must be a multiple of the expert count");
  c10::cuda::CUDAGuard g(dgu.device());
  qw::moe_gate_up_dgrad(bptr(dgu), bptr(w), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, G, E, H, F,
                        bptr_mut(dx), stream());
}

void moe_wgrad(Tensor a, Tensor b, Tensor counts, Tensor offsets, Tensor out, bool accumulate, int64_t segments,
               double alpha) {
  CHECK_CUDA(a); CHECK_CONTIG(a); CHECK_CONTIG(b); CHECK_CONTIG(out);
  const int64_t E = out.size(0), M = out.size(1), N = out.size(2), R = a.size(0);
  TORCH_CHECK(a.size(1) == M && b.size(1) == N && b.size(0) == R, "moe_wgrad shapes");
  TORCH_CHECK(segments >= 1 && counts.numel() == E * segments, "moe_wgrad: counts must hold segments * experts");
  check_groups(counts, offsets, E * segments);
  const bool fp32 = out.scalar_type() == torch::kFloat32;
  c10::cuda::CUDAGuard g(a.device());
  qw::moe_wgrad(bptr(a), bptr(b), counts.data_ptr<int>(), offsets.data_ptr<int>(), R, E, static_cast<int>(segments), M,
                N, out.data_ptr(), fp32, accumulate, static_cast<float>(alpha), stream());
}

// ------------------------------------------------------------------------------------------------ norm / rope
void norm_fwd(Tensor x, OptT delta, OptT x_out, Tensor w, OptT b, Tensor y, OptT mean, Tensor rstd, double eps,
              bool rms) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_CONTIG(y);
  CHECK_DTYPE(w, torch::kFloat32); CHECK_DTYPE(rstd, torch::kFloat32);
  const int H = static_cast<int>(x.size(-1));
  const int64_t rows = x.numel() / H;
  c10::cuda::CUDAGuard g(x.device());
  qw::norm_fwd(bptr(x), optb(delta), optb_mut(x_out), w.data_ptr<float>(), optptr<float>(b), bptr_mut(y),
               mean ? mean->data_ptr<float>() : nullptr, rstd.data_ptr<float>(), rows, H, static_cast<float>(eps), rms,
               stream());
}

int64_t norm_bwd_blocks(int64_t rows) { return qw::norm_bwd_blocks(rows); }

int64_t bias_grad_slabs(int64_t rows) { return qw::bias_grad_slabs(rows); }

// out[c] (+)= sum_r g[r, c] in fp32 (deterministic two-stage reduction); part: [bias_grad_slabs(rows), N] fp32
void bias_grad(Tensor g, Tensor part, Tensor out, bool accumulate) {
  CHECK_CUDA(g); CHECK_ROWS(g); CHECK_DTYPE(out, torch::kFloat32); CHECK_DTYPE(part, torch::kFloat32);
  c10::cuda::CUDAGuard guard(g.device());
  qw::bias_grad(bptr(g), g.stride(0), g.size(0), static_cast<int>(g.size(1)), part.data_ptr<float>(),
                out.data_ptr<float>(), accumulate, stream());
}

void norm_bwd(Tensor dy, Tensor x, Tensor w, OptT mean, Tensor rstd, OptT dres, Tensor dx, Tensor dw_part,
              OptT db_part, Tensor dw, OptT db, bool rms, bool accumulate) {
  CHECK_CUDA(dy); CHECK_CONTIG(dy); CHECK_CONTIG(x); CHECK_CONTIG(dx);
  const int H = static_cast<int>(x.size(-1));
  const int64_t rows = x.numel() / H;
  c10::cuda::CUDAGuard g(x.device());
  qw::norm_bwd(bptr(dy), bptr(x), w.data_ptr<float>(), mean ? mean->data_ptr<float>() : nullptr, rstd.data_ptr<float>(),
               optb(dres), bptr_mut(dx), dw_part.data_ptr<float>(), db_part ? db_part->data_ptr<float>() : nullptr,
               dw.data_ptr<float>(), db ? db->data_ptr<float>() : nullptr, rows, H, rms, accumulate, stream());
}

void rope_apply(Tensor qkv, int64_t heads_rot, int64_t head_dim, int64_t seq, OptT positions, Tensor cos_t,
                Tensor sin_t, bool inverse) {
  CHECK_CUDA(qkv); CHECK_ROWS(qkv);
  CHECK_DTYPE(cos_t, torch::kFloat32); CHECK_DTYPE(sin_t, torch::kFloat32);
  c10::cuda::CUDAGuard g(qkv.device());
  qw::rope_apply(bptr_mut(qkv), qkv.size(0), static_cast<int>(heads_rot), static_cast<int>(head_dim), qkv.stride(0),
                 static_cast<int>(seq), optptr<int>(positions), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                 inverse, stream());
}

// ------------------------------------------------------------------------------------------------ routing
void router_logits(Tensor x, Tensor w, Tensor logits) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DTYPE(w, torch::kFloat32); CHECK_CONTIG(w); CHECK_CONTIG(logits);
  c10::cuda::CUDAGuard g(x.device());
  const int64_t T = x.size(0);
  const int H = static_cast<int>(x.size(1)), E = static_cast<int>(w.size(0));
  if (qw::router_tc_ok(T, H, E)) {  // tensor cores over the bf16 split of Wr (fp32-exact products)
    auto w3 = torch::empty({3 * E, H}, x.options().dtype(torch::kBFloat16));
    auto out3 = torch::empty({T, 3 * E}, x.options().dtype(torch::kFloat32));
    qw::router_logits_tc(bptr(x), w.data_ptr<float>(), T, H, E, logits.data_ptr<float>(), bptr_mut(w3),
                         out3.data_ptr<float>(), stream());
    return;
  }
  qw::router_logits(bptr(x), w.data_ptr<float>(), T, H, E, logits.data_ptr<float>(), stream());
}

void router_topk(Tensor logits, OptT bias, int64_t k, double temperature, Tensor probs, Tensor top_idx, Tensor top_w,
                 Tensor counts) {
  CHECK_CUDA(logits); CHECK_CONTIG(logits);
  c10::cuda::CUDAGuard g(logits.device());
  qw::router_topk(logits.data_ptr<float>(), optptr<float>(bias), logits.size(0), static_cast<int>(logits.size(1)),
                  static_cast<int>(k), static_cast<float>(temperature), probs.data_ptr<float>(), top_idx.data_ptr<int>(),
                  top_w.data_ptr<float>(), counts.data_ptr<int>(), stream());
}

int64_t moe_plan_chunks(int64_t routes) { return qw::moe_plan_chunks(routes); }

void moe_plan(Tensor top_idx, Tensor top_w, Tensor counts, int64_t cap, int64_t slot_rows, Tensor kept, Tensor offsets,
              Tensor uoffsets, Tensor meta, Tensor chunk_hist, Tensor sorted_routes, Tensor route_row) {
  CHECK_CUDA(top_idx);
  const int E = static_cast<int>(counts.numel());
  c10::cuda::CUDAGuard g(top_idx.device());
  qw::moe_plan(top_idx.data_ptr<int>(), top_w.data_ptr<float>(), counts.data_ptr<int>(), top_idx.numel(), E,
               static_cast<int>(std::min<int64_t>(cap, INT32_MAX)), static_cast<int>(slot_rows), kept.data_ptr<int>(),
               offsets.data_ptr<int>(),
               uoffsets.data_ptr<int>(), meta.data_ptr<int>(), chunk_hist.data_ptr<int>(), sorted_routes.data_ptr<int>(),
               route_row.data_ptr<int>(), stream());
}

void moe_permute(Tensor x, int64_t k, Tensor route_row, Tensor top_w, Tensor kept, Tensor offsets, Tensor x_perm,
                 Tensor row_token, Tensor row_w) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_CONTIG(x_perm);
  c10::cuda::CUDAGuard g(x.device());
  qw::moe_permute(bptr(x), route_row.numel(), static_cast<int>(k), static_cast<int>(x.size(1)),
                  route_row.data_ptr<int>(), top_w.data_ptr<float>(), kept.data_ptr<int>(), offsets.data_ptr<int>(),
                  static_cast<int>(kept.numel()), bptr_mut(x_perm), row_token.data_ptr<int>(), row_w.data_ptr<float>(),
                  x_perm.size(0), stream());
}

void moe_pad_zero(Tensor kept, Tensor offsets, Tensor buf) {
  CHECK_CUDA(buf); CHECK_CONTIG(buf);
  c10::cuda::CUDAGuard g(buf.device());
  qw::moe_pad_zero(kept.data_ptr<int>(), offsets.data_ptr<int>(), static_cast<int>(kept.numel()),
                   static_cast<int>(buf.size(1)), bptr_mut(buf), stream());
}

void moe_gather_rows(Tensor src, Tensor row_token, Tensor meta, Tensor dst) {
  CHECK_CUDA(src); CHECK_CONTIG(src); CHECK_CONTIG(dst);
  c10::cuda::CUDAGuard g(src.device());
  qw::moe_gather_rows(bptr(src), row_token.data_ptr<int>(), meta.data_ptr<int>(), dst.size(0),
                      static_cast<int>(dst.size(1)), bptr_mut(dst), stream());
}

void moe_combine(Tensor y, Tensor route_row, Tensor top_w, OptT resid, int64_t k, Tensor out) {
  CHECK_CUDA(y); CHECK_CONTIG(y); CHECK_CONTIG(out);
  c10::cuda::CUDAGuard g(y.device());
  qw::moe_combine(bptr(y), route_row.data_ptr<int>(), top_w.data_ptr<float>(), optb(resid), out.size(0),
                  static_cast<int>(k), static_cast<int>(out.size(1)), bptr_mut(out), y.size(0), stream());
}

void moe_combine_grad(Tensor dx_perm, Tensor route_row, OptT extra, int64_t k, Tensor dx) {
  CHECK_CUDA(dx_perm); CHECK_CONTIG(dx_perm); CHECK_CONTIG(dx);
  c10::cuda::CUDAGuard g(dx.device());
  qw::moe_combine_grad(bptr(dx_perm), route_row.data_ptr<int>(), optptr<float>(extra), dx.size(0), static_cast<int>(k),
                       static_cast<int>(dx.size(1)), bptr_mut(dx), dx_perm.size(0), stream());
}

void moe_route_dw(Tensor partial, Tensor route_row, Tensor d_w) {
  CHECK_CUDA(partial);
  c10::cuda::CUDAGuard g(partial.device());
  qw::moe_route_dw(partial.data_ptr<float>(), static_cast<int>(partial.size(1)), route_row.data_ptr<int>(),
                   route_row.numel(), d_w.data_ptr<float>(), stream());
}

void router_backward(Tensor probs, Tensor top_idx, Tensor top_w, Tensor d_w, OptT d_probs, double temperature,
                     Tensor d_logits) {
  CHECK_CUDA(probs);
  c10::cuda::CUDAGuard g(probs.device());
  qw::router_backward(probs.data_ptr<float>(), top_idx.data_ptr<int>(), top_w.data_ptr<float>(), d_w.data_ptr<float>(),
                      optptr<float>(d_probs), probs.size(0), static_cast<int>(probs.size(1)),
                      static_cast<int>(top_idx.size(1)), static_cast<float>(temperature), d_logits.data_ptr<float>(),
                      stream());
}

void router_dx(Tensor d_logits, Tensor w, Tensor dx) {
  CHECK_CUDA(d_logits); CHECK_CONTIG(d_logits); CHECK_CONTIG(w); CHECK_CONTIG(dx);
  c10::cuda::CUDAGuard g(d_logits.device());
  const int64_t T = d_logits.size(0);
  const int E = static_cast<int>(d_logits.size(1)), H = static_cast<int>(w.size(1));
  if (qw::router_tc_ok(T, H, E)) {
    auto dls = torch::empty({T, 3 * E}, d_logits.options().dtype(torch::kBFloat16));
    auto w3 = torch::empty({3 * E, H}, d_logits.options().dtype(torch::kBFloat16));
    qw::router_dx_tc(d_logits.data_ptr<float>(), w.data_ptr<float>(), T, E, H, dx.data_ptr<float>(), bptr_mut(dls),
                     bptr_mut(w3), stream());
    return;
  }
  qw::router_dx(d_logits.data_ptr<float>(), w.data_ptr<float>(), T, E, H, dx.data_ptr<float>(), stream());
}

int64_t router_dw_split(int64_t T) { return qw::router_dw_split(T); }

void router_dw(Tensor d_logits, Tensor x, Tensor dw, bool accumulate, Tensor workspace) {
  CHECK_CUDA(d_logits); CHECK_CONTIG(d_logits); CHECK_CONTIG(x); CHECK_DTYPE(x, torch::kBFloat16);
  c10::cuda::CUDAGuard g(d_logits.device());
  const int64_t T = d_logits.size(0);
  const int E = static_cast<int>(d_logits.size(1)), H = static_cast<int>(x.size(1));
  if (qw::router_tc_ok(T, H, E)) {
    const int64_t chunks = (T + qw::router_dw_chunk(T, H) - 1) / qw::router_dw_chunk(T, H);
    auto dls = torch::empty({T, 3 * E}, d_logits.options().dtype(torch::kBFloat16));
    auto partial = torch::empty({chunks * 2 * E * H}, d_logits.options().dtype(torch::kFloat32));
    qw::router_dw_tc(d_logits.data_ptr<float>(), bptr(x), T, E, H, dw.data_ptr<float>(), accumulate, bptr_mut(dls),
                     partial.data_ptr<float>(), stream());
    return;
  }
  qw::router_dw(d_logits.data_ptr<float>(), bptr(x), T, E, H, dw.data_ptr<float>(), accumulate,
                workspace.data_ptr<float>(), stream());
}

// ------------------------------------------------------------------------------------------------ optimizer / CE
int64_t adam_chunk_size() { return qw::adam_chunk_size(); }
int64_t adam8_block_size() { return qw::adam8_block_size(); }

static_assert(sizeof(qw::AdamTensor) == 64, "AdamTensor layout is mirrored in Python (8 x 8 bytes)");

void adam_grad_norm(Tensor table, Tensor chunk_tensor, Tensor chunk_start, Tensor partial, OptT extra_sumsq,
                    double max_norm, Tensor norm_out) {
  CHECK_CUDA(table);
  c10::cuda::CUDAGuard g(table.device());
  qw::adam_grad_norm(reinterpret_cast<const qw::AdamTensor*>(table.data_ptr()), chunk_tensor.data_ptr<int>(),
                     chunk_start.data_ptr<int64_t>(), static_cast<int>(chunk_tensor.numel()),
                     partial.data_ptr<double>(), optptr<double>(extra_sumsq), static_cast<float>(max_norm),
                     norm_out.data_ptr<float>(), stream());
}

void adam_sumsq(Tensor table, Tensor chunk_tensor, Tensor chunk_start, Tensor partial) {
  CHECK_CUDA(table);
  c10::cuda::CUDAGuard g(table.device());
  qw::adam_sumsq(reinterpret_cast<const qw::AdamTensor*>(table.data_ptr()), chunk_tensor.data_ptr<int>(),
                 chunk_start.data_ptr<int64_t>(), static_cast<int>(chunk_tensor.numel()), partial.data_ptr<double>(),
                 stream());
}

void adam_step(Tensor table, Tensor chunk_tensor, Tensor chunk_start, double lr, double beta1, double beta2, double eps,
               double weight_decay, int64_t step, OptT clip, bool eight_bit, int64_t small_blocks) {
  CHECK_CUDA(table);
  qw::AdamHyper h;
  h.lr = static_cast<float>(lr);
  h.beta1 = static_cast<float>(beta1);
  h.beta2 = static_cast<float>(beta2);
  h.eps = static_cast<float>(eps);
  h.weight_decay = static_cast<float>(weight_decay);
  h.bias_correction1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  h.bias_correction2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  c10::cuda::CUDAGuard g(table.device());
  qw::adam_step(reinterpret_cast<const qw::AdamTensor*>(table.data_ptr()), chunk_tensor.data_ptr<int>(),
                chunk_start.data_ptr<int64_t>(), static_cast<int>(chunk_tensor.numel()), h, optptr<float>(clip),
                eight_bit, stream(), static_cast<int>(small_blocks));
}

void cross_entropy_chunk(Tensor logits, Tensor labels, double grad_scale, Tensor loss_out, int64_t ignore_index) {
  CHECK_CUDA(logits); CHECK_ROWS(logits); CHECK_DTYPE(labels, torch::kInt64);
  c10::cuda::CUDAGuard g(logits.device());
  qw::cross_entropy_chunk(bptr_mut(logits), logits.size(0), logits.stride(0), static_cast<int>(logits.size(1)),
                          labels.data_ptr<int64_t>(), static_cast<float>(grad_scale), loss_out.data_ptr<float>(),
                          static_cast<int>(ignore_index), stream());
}

void scale_bf16(Tensor x, Tensor scale) {
  CHECK_CUDA(x); CHECK_CONTIG(x);
  c10::cuda::CUDAGuard g(x.device());
  qw::scale_bf16(bptr_mut(x), x.numel(), scale.data_ptr<float>(), stream());
}

// ------------------------------------------------------------------------------------------------ attention
void flash_attn_fwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                    int64_t D, double scale) {
  CHECK_CUDA(q); CHECK_ROWS(q); CHECK_ROWS(k); CHECK_ROWS(v); CHECK_ROWS(o);
  TORCH_CHECK(q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0 && o.stride(0) % 8 == 0,
              "attention rows must be 16-byte aligned");
  c10::cuda::CUDAGuard g(q.device());
  qw::flash_attn_fwd(bptr(q), q.stride(0), bptr(k), k.stride(0), bptr(v), v.stride(0), bptr_mut(o), o.stride(0),
                     lse.data_ptr<float>(), static_cast<int>(B), static_cast<int>(S), static_cast<int>(Hq),
                     static_cast<int>(Hkv), static_cast<int>(D), static_cast<float>(scale), stream());
}

void flash_attn_bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor dout, Tensor lse, Tensor delta, Tensor dq,
                    Tensor dk, Tensor dv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D, double scale) {
  CHECK_CUDA(q); CHECK_ROWS(q); CHECK_ROWS(dout); CHECK_ROWS(dq); CHECK_ROWS(dk); CHECK_ROWS(dv);
  c10::cuda::CUDAGuard g(q.device());
  qw::flash_attn_bwd(bptr(q), q.stride(0), bptr(k), k.stride(0), bptr(v), v.stride(0), bptr(o), o.stride(0),
                     bptr(dout), dout.stride(0), lse.data_ptr<float>(), delta.data_ptr<float>(), bptr_mut(dq),
                     dq.stride(0), bptr_mut(dk), dk.stride(0), bptr_mut(dv), dv.stride(0), static_cast<int>(B),
                     static_cast<int>(S), static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(D),
                     static_cast<float>(scale), stream());
}

// ------------------------------------------------------------------------------------------------ p2p
// peer_bufs / peer_flags: int64 device tensors of raw peer addresses (from the symmetric-memory rendezvous)
void p2p_broadcast(Tensor src, Tensor peer_bufs, Tensor peer_flags, int64_t me, int64_t epoch, Tensor done) {
  CHECK_CUDA(src); CHECK_CONTIG(src);
  c10::cuda::CUDAGuard g(src.device());
  qw::p2p_broadcast(src.data_ptr(), src.numel() * src.element_size(),
                    reinterpret_cast<void* const*>(peer_bufs.data_ptr<int64_t>()),
                    reinterpret_cast<int* const*>(peer_flags.data_ptr<int64_t>()), static_cast<int>(peer_bufs.numel()),
                    static_cast<int>(me), static_cast<int>(epoch), reinterpret_cast<unsigned int*>(done.data_ptr<int>()),
                    stream());
}

void p2p_push(Tensor src, int64_t block_bytes, Tensor peer_bufs, Tensor peer_flags, int64_t me, int64_t epoch,
              Tensor done) {
  CHECK_CUDA(src); CHECK_CONTIG(src);
  TORCH_CHECK(src.numel() * src.element_size() == block_bytes * peer_bufs.numel(), "p2p_push: src size");
  c10::cuda::CUDAGuard g(src.device());
  qw::p2p_push(src.data_ptr(), block_bytes, reinterpret_cast<void* const*>(peer_bufs.data_ptr<int64_t>()),
               reinterpret_cast<int* const*>(peer_flags.data_ptr<int64_t>()), static_cast<int>(peer_bufs.numel()),
               static_cast<int>(me), static_cast<int>(epoch), reinterpret_cast<unsigned int*>(done.data_ptr<int>()),
               stream());
}

void p2p_wait(Tensor flags, int64_t world, int64_t epoch, double timeout_s) {
  CHECK_CUDA(flags);
  c10::cuda::CUDAGuard g(flags.device());
  qw::p2p_wait(flags.data_ptr<int>(), static_cast<int>(world), static_cast<int>(epoch), timeout_s, stream());
}

// ------------------------------------------------------------------------------------------------ fused EP exchange
// peer / peer_flags: int64 device tensors of every rank's buffer / flag base addresses (symmetric memory)
void ep_dispatch(Tensor x, Tensor route_row, OptT top_w, OptT kept, int64_t k, int64_t E, int64_t local, int64_t slot,
                 int64_t me, Tensor peer, int64_t w_off, int64_t c_off, Tensor peer_flags, int64_t epoch, Tensor done) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DTYPE(x, torch::kBFloat16);
  c10::cuda::CUDAGuard g(x.device());
  qw::ep_dispatch(bptr(x), x.size(0), static_cast<int>(k), static_cast<int>(x.size(1)), route_row.data_ptr<int>(),
                  optptr<float>(top_w), optptr<int>(kept), static_cast<int>(E), static_cast<int>(local),
                  static_cast<int>(slot), static_cast<int>(me), static_cast<int>(peer.numel()),
                  reinterpret_cast<uint8_t* const*>(peer.data_ptr<int64_t>()), w_off, c_off,
                  reinterpret_cast<int* const*>(peer_flags.data_ptr<int64_t>()), static_cast<int>(epoch),
                  reinterpret_cast<unsigned int*>(done.data_ptr<int>()), stream());
}

void ep_pad(Tensor counts, int64_t slot, Tensor rows, OptT w) {
  CHECK_CUDA(rows); CHECK_ROWS(rows);
  c10::cuda::CUDAGuard g(rows.device());
  qw::ep_pad(counts.data_ptr<int>(), static_cast<int>(counts.numel()), static_cast<int>(slot),
             static_cast<int>(rows.size(1)), bptr_mut(rows), w ? w->data_ptr<float>() : nullptr, stream());
}

void ep_signal(Tensor peer_flags, int64_t me, int64_t epoch) {
  c10::cuda::CUDAGuard g(peer_flags.device());
  qw::ep_signal(reinterpret_cast<int* const*>(peer_flags.data_ptr<int64_t>()), static_cast<int>(peer_flags.numel()),
                static_cast<int>(me), static_cast<int>(epoch), stream());
}


// ------------------------------------------------------------------------------------------------ fused ZeRO
int64_t zero_rs_blocks(int64_t per) { return qw::zero_rs_blocks(per); }

// peers: int64 tensor of every rank's flat staging (gradients) or parameter buffer; dtype 0 fp32, 1 bf16
void zero_reduce_scatter(Tensor peers, int64_t dtype, int64_t start, Tensor shard, Tensor partial) {
  CHECK_CUDA(shard); CHECK_DTYPE(shard, torch::kFloat32); CHECK_DTYPE(partial, torch::kFloat64);
  c10::cuda::CUDAGuard g(shard.device());
  qw::zero_reduce_scatter(reinterpret_cast<const void* const*>(peers.data_ptr<int64_t>()),
                          static_cast<int>(peers.numel()), static_cast<int>(dtype), start, shard.numel(),
                          shard.data_ptr<float>(), partial.data_ptr<double>(), stream());
}

void zero_adamw_gather(Tensor master, Tensor m, Tensor v, Tensor grad, OptT clip, double lr, double beta1, double beta2,
                       double eps, double weight_decay, int64_t step, Tensor peers, int64_t dtype, int64_t start,
                       int64_t valid) {
  CHECK_CUDA(master);
  qw::AdamHyper h;
  h.lr = static_cast<float>(lr);
  h.beta1 = static_cast<float>(beta1);
  h.beta2 = static_cast<float>(beta2);
  h.eps = static_cast<float>(eps);
  h.weight_decay = static_cast<float>(weight_decay);
  h.bias_correction1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  h.bias_correction2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  c10::cuda::CUDAGuard g(master.device());
  qw::zero_adamw_gather(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr<float>(),
                        optptr<float>(clip), h, reinterpret_cast<void* const*>(peers.data_ptr<int64_t>()),
                        static_cast<int>(peers.numel()), static_cast<int>(dtype), start, master.numel(), valid,
                        stream());
}

// ------------------------------------------------------------------------------------------------ decode
// w: [G, rows, ...] packed weights (uint8 / int8 / bf16 viewed as bytes), scales: fp16 or None (bf16 weights)
void grouped_gemv(Tensor x, Tensor w, OptT scales, int64_t N, int64_t K, int64_t group, int64_t fmt, bool swiglu,
                  OptT tok, OptT off, OptT cnt, int64_t groups, int64_t dense_rows, Tensor out, bool out_by_route,
                  OptT bias, OptT resid, OptT active) {
  CHECK_CUDA(x); CHECK_ROWS(x); CHECK_CONTIG(w); CHECK_ROWS(out);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kBFloat16);
  if (scales) TORCH_CHECK(scales->scalar_type() == torch::kFloat16 && scales->is_contiguous());
  const int64_t w_group_bytes = w.numel() * w.element_size() / groups;
  const int64_t s_group = scales ? scales->numel() / groups : 0;
  c10::cuda::CUDAGuard g(x.device());
  qw::grouped_gemv(bptr(x), x.stride(0), w.data_ptr(), scales ? scales->data_ptr() : nullptr, w_group_bytes, s_group,
                   static_cast<int>(N), static_cast<int>(K), static_cast<int>(group), static_cast<int>(fmt), swiglu,
                   optptr<int>(tok), optptr<int>(off), optptr<int>(cnt), static_cast<int>(groups),
                   static_cast<int>(dense_rows), bptr_mut(out), out.stride(0), out_by_route, optptr<float>(bias),
                   optb(resid), resid ? resid->stride(0) : 0, optptr<int>(active),
                   active ? static_cast<int>(active->numel()) : 0, stream());
}

void decode_route(Tensor x, Tensor wr, OptT ebias, int64_t k, double temperature, Tensor logits, Tensor cnt, Tensor off,
                  Tensor order, Tensor route_slot, Tensor top_w, Tensor active, Tensor ticket) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DTYPE(wr, torch::kFloat32);
  c10::cuda::CUDAGuard g(x.device());
  qw::decode_route(bptr(x), wr.data_ptr<float>(), optptr<float>(ebias), static_cast<int>(x.size(0)),
                   static_cast<int>(x.size(1)), static_cast<int>(wr.size(0)), static_cast<int>(k),
                   static_cast<float>(temperature), logits.data_ptr<float>(), cnt.data_ptr<int>(), off.data_ptr<int>(),
                   order.data_ptr<int>(), route_slot.data_ptr<int>(), top_w.data_ptr<float>(), active.data_ptr<int>(),
                   ticket.data_ptr<int>(), stream());
}

int64_t decode_attn_chunks(int64_t Lmax) { return qw::decode_attn_chunks(static_cast<int>(Lmax)); }

void decode_attention(Tensor q, Tensor kc, Tensor vc, Tensor lens, double scale, Tensor part_o, Tensor part_ml,
                      Tensor tickets, Tensor out) {
  CHECK_CUDA(q); CHECK_CONTIG(q); CHECK_CONTIG(kc); CHECK_CONTIG(vc); CHECK_CONTIG(out);
  const int B = static_cast<int>(kc.size(0)), Hkv = static_cast<int>(kc.size(1)), Lmax = static_cast<int>(kc.size(2));
  const int D = static_cast<int>(kc.size(3)), Hq = static_cast<int>(q.size(1));
  c10::cuda::CUDAGuard g(q.device());
  qw::decode_attention(bptr(q), bptr(kc), bptr(vc), lens.data_ptr<int>(), B, Hq, Hkv, D, Lmax,
                       static_cast<float>(scale), part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                       tickets.data_ptr<int>(), bptr_mut(out), stream());
}

// tokens given: the input row is tok_emb[tokens[t]] (+ pos_emb[positions[t]]); else x[t]. y given: add the MoE output
// sum_j top_w[t, j] * y[slot[t, j]]. Writes the residual to x_out (optional) and the normalised row to n_out.
void decode_combine_norm(OptT x, OptT tokens, OptT tok_emb, OptT pos_emb, OptT positions, OptT y, OptT slot,
                         OptT top_w, int64_t k, Tensor w, OptT bias, double eps, bool rms, OptT x_out, Tensor n_out) {
  CHECK_CUDA(n_out); CHECK_CONTIG(n_out); CHECK_DTYPE(w, torch::kFloat32);
  if (x) { CHECK_CONTIG((*x)); }
  if (tokens) TORCH_CHECK(tokens->scalar_type() == torch::kInt64 && tok_emb && positions);
  c10::cuda::CUDAGuard g(n_out.device());
  qw::decode_combine_norm(optb(x), tokens ? tokens->data_ptr<int64_t>() : nullptr, optb(tok_emb), optb(pos_emb),
                          optptr<int>(positions), optb(y), optptr<int>(slot), optptr<float>(top_w),
                          static_cast<int>(k), static_cast<int>(n_out.size(0)), static_cast<int>(n_out.size(1)),
                          w.data_ptr<float>(), optptr<float>(bias), static_cast<float>(eps), rms, optb_mut(x_out),
                          bptr_mut(n_out), stream());
}

// expert-parallel decode: routing over every expert, active list restricted to this rank's [first, first + local)
void decode_route_local(Tensor x, Tensor wr, OptT ebias, int64_t k, double temperature, Tensor logits, Tensor cnt,
                        Tensor off, Tensor order, Tensor route_slot, Tensor top_w, Tensor active, Tensor ticket,
                        int64_t first, int64_t local) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DTYPE(wr, torch::kFloat32);
  TORCH_CHECK(first >= 0 && local > 0 && first + local <= wr.size(0), "decode_route_local: expert range");
  c10::cuda::CUDAGuard g(x.device());
  qw::decode_route(bptr(x), wr.data_ptr<float>(), optptr<float>(ebias), static_cast<int>(x.size(0)),
                   static_cast<int>(x.size(1)), static_cast<int>(wr.size(0)), static_cast<int>(k),
                   static_cast<float>(temperature), logits.data_ptr<float>(), cnt.data_ptr<int>(), off.data_ptr<int>(),
                   order.data_ptr<int>(), route_slot.data_ptr<int>(), top_w.data_ptr<float>(), active.data_ptr<int>(),
                   ticket.data_ptr<int>(), stream(), static_cast<int>(first), static_cast<int>(local));
}

// norm of x + sum over ranks of the expert-parallel partial MoE outputs (plane of `layer` for the current step)
void decode_combine_norm_parts(Tensor x, Tensor parts, Tensor step, int64_t layer, int64_t layers, int64_t world,
                               int64_t tstride, Tensor w, OptT bias, double eps, bool rms, OptT x_out, Tensor n_out) {
  CHECK_CUDA(n_out); CHECK_CONTIG(n_out); CHECK_CONTIG(x); CHECK_DTYPE(w, torch::kFloat32);
  CHECK_DTYPE(parts, torch::kFloat32); CHECK_DTYPE(step, torch::kInt32);
  TORCH_CHECK(parts.numel() >= 2 * layers * world * tstride * n_out.size(1), "decode_combine_norm_parts: planes");
  c10::cuda::CUDAGuard g(n_out.device());
  qw::decode_combine_norm(bptr(x), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0,
                          static_cast<int>(n_out.size(0)), static_cast<int>(n_out.size(1)), w.data_ptr<float>(),
                          optptr<float>(bias), static_cast<float>(eps), rms, optb_mut(x_out), bptr_mut(n_out),
                          stream(), parts.data_ptr<float>(), step.data_ptr<int>(), static_cast<int>(layer),
                          static_cast<int>(layers), static_cast<int>(world), static_cast<int>(tstride));
}

void dequant_rows(Tensor q, Tensor scales, int64_t K, int64_t group, int64_t fmt, Tensor out) {
  CHECK_CUDA(q); CHECK_CONTIG(q); CHECK_CONTIG(scales); CHECK_CONTIG(out);
  TORCH_CHECK(scales.scalar_type() == torch::kFloat16 && out.scalar_type() == torch::kBFloat16, "dequant_rows dtypes");
  TORCH_CHECK(fmt == 1 || fmt == 2, "dequant_rows: fmt 1 (int8) or 2 (int4)");
  const int64_t rows = out.numel() / K;
  TORCH_CHECK(q.numel() == rows * (fmt == 2 ? K / 2 : K), "dequant_rows: packed size");
  c10::cuda::CUDAGuard g(q.device());
  qw::dequant_rows(q.data_ptr(), scales.data_ptr(), rows, static_cast<int>(K), static_cast<int>(group),
                   static_cast<int>(fmt), bptr_mut(out), stream());
}

void ep_decode_tick(Tensor step) {
  CHECK_CUDA(step); CHECK_DTYPE(step, torch::kInt32);
  c10::cuda::CUDAGuard g(step.device());
  qw::ep_decode_tick(step.data_ptr<int>(), stream());
}

void ep_decode_push(Tensor y, Tensor slot, Tensor top_w, int64_t k, int64_t tstride, Tensor peers, int64_t plane_floats,
                    int64_t layer, int64_t layers, int64_t me, Tensor peer_flags, Tensor step, Tensor done) {
  CHECK_CUDA(y); CHECK_CONTIG(y); CHECK_DTYPE(peers, torch::kInt64); CHECK_DTYPE(peer_flags, torch::kInt64);
  const int T = static_cast<int>(top_w.size(0));
  TORCH_CHECK(T <= tstride, "ep_decode_push: more tokens than the exchange planes hold");
  c10::cuda::CUDAGuard g(y.device());
  qw::ep_decode_push(bptr(y), slot.data_ptr<int>(), top_w.data_ptr<float>(), static_cast<int>(k), T,
                     static_cast<int>(y.size(1)), static_cast<int>(tstride),
                     reinterpret_cast<float* const*>(peers.data_ptr<int64_t>()), plane_floats, static_cast<int>(layer),
                     static_cast<int>(layers), static_cast<int>(me), static_cast<int>(peers.numel()),
                     reinterpret_cast<int* const*>(peer_flags.data_ptr<int64_t>()), step.data_ptr<int>(),
                     reinterpret_cast<unsigned int*>(done.data_ptr<int>()), stream());
}

void ep_decode_wait(Tensor flags, int64_t world, Tensor step, int64_t layer, int64_t layers, double timeout_s) {
  CHECK_CUDA(flags); CHECK_DTYPE(flags, torch::kInt32);
  c10::cuda::CUDAGuard g(flags.device());
  qw::ep_decode_wait(flags.data_ptr<int>(), static_cast<int>(world), step.data_ptr<int>(), static_cast<int>(layer),
                     static_cast<int>(layers), timeout_s, stream());
}

void decode_attention_rope(Tensor qkv, Tensor pos, Tensor cos_t, Tensor sin_t, bool rope, Tensor kc, Tensor vc,
                           int64_t Hq, double scale, Tensor part_o, Tensor part_ml, Tensor tickets, Tensor out) {
  CHECK_CUDA(qkv); CHECK_CONTIG(qkv); CHECK_CONTIG(kc); CHECK_CONTIG(vc); CHECK_CONTIG(out);
  const int B = static_cast<int>(qkv.size(0)), Hkv = static_cast<int>(kc.size(1)), Lmax = static_cast<int>(kc.size(2));
  const int D = static_cast<int>(kc.size(3));
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * D, "decode_attention_rope: qkv width");
  TORCH_CHECK(kc.size(0) >= B && pos.numel() >= B, "decode_attention_rope: batch");
  c10::cuda::CUDAGuard g(qkv.device());
  qw::decode_attention_rope(bptr(qkv), pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), rope,
                            bptr_mut(kc), bptr_mut(vc), B, static_cast<int>(Hq), Hkv, D, Lmax,
                            static_cast<float>(scale), part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                            tickets.data_ptr<int>(), bptr_mut(out), stream());
}

void rope_append(Tensor qkv, Tensor pos, int64_t Hq, int64_t Hkv, Tensor cos_t, Tensor sin_t, bool rope, Tensor q_out,
                 Tensor kc, Tensor vc) {
  CHECK_CUDA(qkv); CHECK_CONTIG(qkv);
  const int B = static_cast<int>(qkv.size(0)), D = static_cast<int>(kc.size(3)), Lmax = static_cast<int>(kc.size(2));
  c10::cuda::CUDAGuard g(qkv.device());
  qw::rope_append(bptr(qkv), pos.data_ptr<int>(), B, static_cast<int>(Hq), static_cast<int>(Hkv), D, Lmax,
                  cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), rope, bptr_mut(q_out), bptr_mut(kc), bptr_mut(vc),
                  stream());
}

// ------------------------------------------------------------------------------------------------ status
int64_t read_status(bool clear) {
  int s = qw::gemm_status(clear);
  int t;
  if ((t = qw::norm_status(clear)) && !s) s = t;
  if ((t = qw::routing_status(clear)) && !s) s = t;
  if ((t = qw::optim_status(clear)) && !s) s = t;
  if ((t = qw::attention_status(clear)) && !s) s = t;
  if ((t = qw::attention_tc_status(clear)) && !s) s = t;
  if ((t = qw::attention_fwd_tc_status(clear)) && !s) s = t;
  if ((t = qw::ep_status(clear)) && !s) s = t;
  if ((t = qw::ep_decode_status(clear)) && !s) s = t;
  if ((t = qw::p2p_status(clear)) && !s) s = t;
  if ((t = qw::tp_status(clear)) && !s) s = t;
  if ((t = qw::decode_status(clear)) && !s) s = t;
  return s;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "QuantaWeave-B200 sm_100a kernels";
  m.def("linear_fwd", &linear_fwd);
  m.def("linear_fwd_peer", &linear_fwd_peer);
  m.def("linear_dgrad_peer", &linear_dgrad_peer);
  m.def("tp_reduce_bcast", &tp_reduce_bcast);
  m.def("tp_reduce_rows", &tp_reduce_rows);
  m.def("linear_dgrad", &linear_dgrad);
  m.def("linear_wgrad", &linear_wgrad);
  m.def("moe_gate_up_fwd", &moe_gate_up_fwd);
  m.def("moe_down_fwd", &moe_down_fwd);
  m.def("moe_down_bwd", &moe_down_bwd);
  m.def("moe_gate_up_dgrad", &moe_gate_up_dgrad);
  m.def("moe_down_fwd_peer", &moe_down_fwd_peer);
  m.def("moe_gate_up_dgrad_peer", &moe_gate_up_dgrad_peer);
  m.def("moe_wgrad", &moe_wgrad, py::arg("a"), py::arg("b"), py::arg("counts"), py::arg("offsets"), py::arg("out"),
        py::arg("accumulate"), py::arg("segments") = 1, py::arg("alpha") = 1.0);
  m.def("moe_dw_tiles", [](int64_t F) { return static_cast<int64_t>(qw::moe_dw_tiles(F)); });
  m.def("norm_fwd", &norm_fwd);
  m.def("norm_bwd_blocks", &norm_bwd_blocks);
  m.def("norm_bwd", &norm_bwd);
  m.def("rope_apply", &rope_apply);
  m.def("router_logits", &router_logits);
  m.def("router_topk", &router_topk);
  m.def("moe_plan_chunks", &moe_plan_chunks);
  m.def("moe_plan", &moe_plan);
  m.def("moe_permute", &moe_permute);
  m.def("moe_pad_zero", &moe_pad_zero);
  m.def("moe_gather_rows", &moe_gather_rows);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_grad", &moe_combine_grad);
  m.def("moe_route_dw", &moe_route_dw);
  m.def("router_backward", &router_backward);
  m.def("router_dx", &router_dx);
  m.def("router_dw_split", &router_dw_split);
  m.def("router_dw", &router_dw);
  m.def("adam_chunk_size", &adam_chunk_size);
  m.def("adam8_block_size", &adam8_block_size);
  m.def("adam_grad_norm", &adam_grad_norm);
  m.def("adam_sumsq", &adam_sumsq);
  m.def("adam_step", &adam_step, py::arg("table"), py::arg("chunk_tensor"), py::arg("chunk_start"), py::arg("lr"),
        py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("weight_decay"), py::arg("step"), py::arg("clip"),
        py::arg("eight_bit"), py::arg("small_blocks") = 0);
  m.def("cross_entropy_chunk", &cross_entropy_chunk);
  m.def("scale_bf16", &scale_bf16);
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("grouped_gemv", &grouped_gemv);
  m.def("decode_attn_chunks", &decode_attn_chunks);
  m.def("decode_route", &decode_route);
  m.def("decode_attention", &decode_attention);
  m.def("rope_append", &rope_append);
  m.def("decode_attention_rope", &decode_attention_rope);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("zero_rs_blocks", &zero_rs_blocks);
  m.def("zero_reduce_scatter", &zero_reduce_scatter);
  m.def("zero_adamw_gather", &zero_adamw_gather);
  m.def("ep_pad", &ep_pad);
  m.def("ep_signal", &ep_signal);
  m.def("bias_grad_slabs", &bias_grad_slabs);
  m.def("bias_grad", &bias_grad);
  m.def("decode_combine_norm", &decode_combine_norm);
  m.def("decode_combine_norm_parts", &decode_combine_norm_parts);
  m.def("decode_route_local", &decode_route_local);
  m.def("ep_decode_tick", &ep_decode_tick);
  m.def("dequant_rows", &dequant_rows);
  m.def("ep_decode_push", &ep_decode_push);
  m.def("ep_decode_wait", &ep_decode_wait);
  m.def("p2p_push", &p2p_push);
  m.def("p2p_broadcast", &p2p_broadcast);
  m.def("p2p_wait", &p2p_wait);
  m.def("read_status", &read_status, py::arg("clear") = true);
  m.def("attn_bwd_trace", [](c10::optional<torch::Tensor> buf) {
    if (buf) {
      TORCH_CHECK(buf->is_cuda() && buf->dtype() == torch::kInt64 && buf->numel() >= 2 * 32 * 16 && buf->is_contiguous(),
                  "attn_bwd_trace: a contiguous CUDA int64 tensor of at least 1024 elements");
      qw::attn_bwd_trace(buf->data_ptr());
    } else {
      qw::attn_bwd_trace(nullptr);
    }
  });
  m.def("attn_fwd_trace", [](c10::optional<torch::Tensor> buf) {
    if (buf) {
      TORCH_CHECK(buf->is_cuda() && buf->dtype() == torch::kInt64 && buf->numel() >= 32 * 2 * 8 && buf->is_contiguous(),
                  "attn_fwd_trace: a contiguous CUDA int64 tensor of at least 512 elements");
      qw::attn_fwd_trace(buf->data_ptr());
    } else {
      qw::attn_fwd_trace(nullptr);
    }
  });
  m.def("gemm_trace", [](c10::optional<torch::Tensor> buf) {
    if (buf) {
      TORCH_CHECK(buf->is_cuda() && buf->dtype() == torch::kInt64 && buf->numel() >= 64 * 8 && buf->is_contiguous(),
                  "gemm_trace: a contiguous CUDA int64 tensor of at least 512 elements");
      qw::gemm_trace(buf->data_ptr());
    } else {
      qw::gemm_trace(nullptr);
    }
  });
}
