// Torch glue of the sequence-parallel collectives (sp_comm.cu, the GEMM modes of gemm_bf16.cu and the
// waiting assignment builder of router.cu): argument checks and the SpSync bundle.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "launch.h"
#include "ops.h"

#define B200_SP_CHECK(cond, msg) TORCH_CHECK(cond, "sp: ", msg)
#define B200_SP_LAUNCH(expr)                                                                       \
  do {                                                                                             \
    cudaError_t _e = (expr);                                                                       \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));                      \
  } while (0)

namespace b200 {

static inline cudaStream_t sp_stream() { return at::cuda::getCurrentCUDAStream(); }

// peers: int64 [world] symmetric buffer bases (device); state: int32 [kSpChannels * 4] (device, local);
// status: int32 device word.
static SpSync make_sync(const at::Tensor& peers, int64_t rank, at::Tensor& state, const at::Tensor& status,
                        double timeout_s) {
  B200_SP_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong && peers.dim() == 1, "peers int64 [world]");
  B200_SP_CHECK(state.is_cuda() && state.scalar_type() == at::kInt && state.numel() >= kSpChannels * 4,
                "state int32 [16]");
  B200_SP_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "status int32");
  const int world = (int)peers.numel();
  B200_SP_CHECK(world >= 1 && world <= kSpMaxRanks && rank >= 0 && rank < world, "rank / world");
  SpSync s{};
  s.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  s.rank = (int)rank;
  s.world = world;
  s.state = reinterpret_cast<uint32_t*>(state.data_ptr<int>());
  s.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  s.timeout_ns = (uint64_t)(timeout_s * 1e9);
  return s;
}

static void check_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                  t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "sp: ", name, " must be bf16 [rows, H] with 16-byte aligned rows");
}

void sp_residual_norm_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status,
                         double timeout_s, int64_t src, const c10::optional<at::Tensor>& x,
                         const c10::optional<at::Tensor>& add, const c10::optional<at::Tensor>& dmask,
                         int64_t rs_off, int64_t comb_off, int64_t ag_off, at::Tensor& residual, const at::Tensor& w,
                         double eps, const c10::optional<at::Tensor>& out, bool ag) {
  check_rows(residual, "residual");
  B200_SP_CHECK(residual.is_contiguous(), "residual contiguous");
  const int Tr = (int)residual.size(0), H = (int)residual.size(1);
  B200_SP_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.numel() == H, "norm weight bf16 [H]");
  c10::cuda::CUDAGuard g(residual.device());
  SpNormArgs a{};
  a.s = make_sync(peers, rank, state, status, timeout_s);
  a.src = (int)src;
  if (x.has_value()) {
    check_rows(*x, "x");
    B200_SP_CHECK(x->size(0) == Tr && x->size(1) == H, "x [Tr, H]");
    a.x = reinterpret_cast<const __nv_bfloat16*>(x->data_ptr());
    a.ld_x = x->stride(0);
  }
  if (add.has_value()) {
    check_rows(*add, "add");
    B200_SP_CHECK(add->is_contiguous() && add->size(0) == Tr && add->size(1) == H, "add [Tr, H]");
    a.add = reinterpret_cast<const __nv_bfloat16*>(add->data_ptr());
  }
  if (dmask.has_value()) {
    B200_SP_CHECK(dmask->scalar_type() == at::kInt && dmask->numel() >= Tr, "dmask int32 [Tr]");
    a.dmask = reinterpret_cast<const uint32_t*>(dmask->data_ptr<int>());
  }
  a.rs_off = rs_off;
  a.comb_off = comb_off;
  a.ag_off = ag_off;
  a.residual = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.eps = (float)eps;
  if (out.has_value()) {
    check_rows(*out, "out");
    B200_SP_CHECK(out->size(0) == Tr && out->size(1) == H, "out [Tr, H]");
    a.out = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    a.ld_out = out->stride(0);
  }
  a.ag = ag ? 1 : 0;
  a.Tr = Tr;
  a.H = H;
  B200_SP_LAUNCH(sp_residual_norm(a, sp_stream()));
}

void sp_route_dispatch_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status,
                          double timeout_s, const at::Tensor& logits, const at::Tensor& h, int64_t k, int64_t mode,
                          const c10::optional<at::Tensor>& bias, double scale, bool renorm, int64_t e_per_rank,
                          int64_t rows_off, int64_t ids_off, int64_t w_off, at::Tensor& dmask,
                          const c10::optional<at::Tensor>& ids_local, const c10::optional<at::Tensor>& w_local) {
  check_rows(h, "h");
  B200_SP_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.is_contiguous() && logits.dim() == 2 &&
                    logits.size(0) == h.size(0),
                "logits fp32 [Tr, E]");
  const int Tr = (int)h.size(0);
  B200_SP_CHECK(dmask.scalar_type() == at::kInt && dmask.numel() >= Tr, "dmask int32 [Tr]");
  c10::cuda::CUDAGuard g(h.device());
  SpDispatchArgs a{};
  a.s = make_sync(peers, rank, state, status, timeout_s);
  a.logits = logits.data_ptr<float>();
  a.h = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  a.ld_h = h.stride(0);
  a.E = (int)logits.size(1);
  a.k = (int)k;
  a.mode = (int)mode;
  a.renorm = renorm ? 1 : 0;
  if (bias.has_value()) {
    B200_SP_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == a.E && bias->is_contiguous(), "bias fp32 [E]");
    a.bias = bias->data_ptr<float>();
  }
  a.scale = (float)scale;
  a.e_per_rank = (int)e_per_rank;
  B200_SP_CHECK((int64_t)a.e_per_rank * a.s.world == a.E, "experts must divide over the ranks");
  a.rows_off = rows_off;
  a.ids_off = ids_off;
  a.w_off = w_off;
  a.dmask = reinterpret_cast<uint32_t*>(dmask.data_ptr<int>());
  if (ids_local.has_value()) {
    B200_SP_CHECK(w_local.has_value() && ids_local->scalar_type() == at::kInt && ids_local->numel() >= (int64_t)Tr * k &&
                      w_local->scalar_type() == at::kFloat && w_local->numel() >= (int64_t)Tr * k,
                  "ids_local int32 / w_local fp32 [Tr, k]");
    a.ids_local = ids_local->data_ptr<int>();
    a.w_local = w_local->data_ptr<float>();
  }
  a.Tr = Tr;
  a.H = (int)h.size(1);
  B200_SP_LAUNCH(sp_route_dispatch(a, sp_stream()));
}

void sp_combine_push_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status, double timeout_s,
                        const at::Tensor& y, const at::Tensor& slot_of, const at::Tensor& sorted_weight, int64_t k,
                        int64_t comb_off, int64_t Tr, int64_t H, int64_t channel) {
  B200_SP_CHECK(y.is_cuda() && y.scalar_type() == at::kFloat && y.dim() == 2 && y.stride(1) == 1 && y.size(1) >= H,
                "y fp32 [assignments, >= H]");
  B200_SP_CHECK(slot_of.scalar_type() == at::kInt && slot_of.is_contiguous() && slot_of.numel() >= peers.numel() * Tr * k,
                "slot_of int32 [world * Tr, k]");
  B200_SP_CHECK(sorted_weight.scalar_type() == at::kFloat, "sorted_weight fp32");
  c10::cuda::CUDAGuard g(y.device());
  SpCombineArgs a{};
  a.s = make_sync(peers, rank, state, status, timeout_s);
  a.y = y.data_ptr<float>();
  a.ld_y = y.stride(0);
  a.slot_of = slot_of.data_ptr<int>();
  a.sorted_weight = sorted_weight.data_ptr<float>();
  a.k = (int)k;
  a.comb_off = comb_off;
  a.Tr = (int)Tr;
  a.H = (int)H;
  a.channel = (int)channel;
  B200_SP_LAUNCH(sp_combine_push(a, sp_stream()));
}

void sp_wait_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status, double timeout_s,
                int64_t channel) {
  c10::cuda::CUDAGuard g(state.device());
  B200_SP_LAUNCH(sp_wait(make_sync(peers, rank, state, status, timeout_s), (int)channel, sp_stream()));
}

void gemm_sp_op(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& out, at::Tensor& status,
                int64_t splits, const at::Tensor& peers, int64_t rank, at::Tensor& state, double timeout_s, int64_t mode,
                int64_t rs_off, int64_t rows_per_rank) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm_sp: bf16 operands");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1) && x.stride(1) == 1 && w.stride(1) == 1,
              "gemm_sp: shapes");
  c10::cuda::CUDAGuard g(x.device());
  GemmSpArgs a{};
  a.g.x = x.data_ptr();
  a.g.ldx = x.stride(0);
  a.g.w = w.data_ptr();
  a.g.ldw = w.stride(0);
  a.g.M = x.size(0);
  a.g.N = w.size(0);
  a.g.K = x.size(1);
  a.g.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  if (mode == 2) {
    TORCH_CHECK(out.has_value() && out->size(0) == x.size(0) && out->size(1) == w.size(0) && out->stride(1) == 1,
                "gemm_sp: all-gather mode writes out [M, N]");
    TORCH_CHECK(out->scalar_type() == at::kBFloat16 || out->scalar_type() == at::kFloat, "gemm_sp: out bf16 / fp32");
    a.g.c = out->data_ptr();
    a.g.ldc = out->stride(0);
    a.g.out_f32 = out->scalar_type() == at::kFloat ? 1 : 0;
  }
  a.g.splits = gemm_bf16_splits(a.g.M, a.g.N, a.g.K, (int)splits);
  at::Tensor partial;
  if (mode == 2 && gemm_bf16_uses_partial(a.g.M, a.g.splits)) {
    partial = at::empty({(int64_t)a.g.splits * a.g.M * a.g.N}, x.options().dtype(at::kFloat));
    a.g.partial = partial.data_ptr<float>();
    a.g.partial_cap = partial.numel();
  }
  a.mode = (int)mode;
  a.sp = make_sync(peers, rank, state, status, timeout_s);
  a.rs_off = rs_off;
  a.rows_per_rank = (int)rows_per_rank;
  B200_SP_LAUNCH(gemm_bf16_sp(a, sp_stream()));
}

void moe_build_assignments_sp_op(const at::Tensor& ids, const at::Tensor& weights,
                                 const c10::optional<at::Tensor>& expert_map, int64_t E_local, int64_t tile_rows,
                                 at::Tensor& sorted_token, at::Tensor& sorted_weight, at::Tensor& slot_of,
                                 at::Tensor& items, at::Tensor& num_items, at::Tensor& expert_offsets,
                                 const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status,
                                 double timeout_s) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && ids.dim() == 2 && ids.is_contiguous(),
              "build_sp: ids int32 [rows, k]");
  TORCH_CHECK(weights.scalar_type() == at::kFloat && weights.sizes() == ids.sizes(), "build_sp: weights");
  const int T = ids.size(0), k = ids.size(1);
  TORCH_CHECK(sorted_token.numel() >= (int64_t)T * k && sorted_weight.numel() >= (int64_t)T * k &&
                  slot_of.numel() >= (int64_t)T * k && items.dim() == 2 && items.size(1) == 4 &&
                  expert_offsets.numel() >= E_local + 1,
              "build_sp: output buffers");
  c10::cuda::CUDAGuard g(ids.device());
  const SpSync s = make_sync(peers, rank, state, status, timeout_s);
  B200_SP_LAUNCH(moe_build_assignments(
      ids.data_ptr<int>(), weights.data_ptr<float>(), T, k,
      expert_map.has_value() ? expert_map->data_ptr<int>() : nullptr,
      expert_map.has_value() ? (int)expert_map->numel() : (int)E_local, (int)E_local, (int)tile_rows,
      sorted_token.data_ptr<int>(), sorted_weight.data_ptr<float>(), slot_of.data_ptr<int>(),
      reinterpret_cast<int4*>(items.data_ptr<int>()), num_items.data_ptr<int>(), expert_offsets.data_ptr<int>(),
      (int)items.size(0), sp_stream(), &s));
}

// out[b] = x[b] . w[b]^T over a batch of matrices (3-D views with unit inner stride; any outer strides
// that are multiples of 8 elements).
void gemm_batched_op(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const at::Tensor& status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "gemm_batched: bf16 tensors");
  TORCH_CHECK(x.dim() == 3 && w.dim() == 3 && out.dim() == 3, "gemm_batched: [B, M, K] x [B, N, K] -> [B, M, N]");
  const int64_t B = x.size(0), M = x.size(1), K = x.size(2), N = w.size(1);
  TORCH_CHECK(w.size(0) == B && w.size(2) == K && out.size(0) == B && out.size(1) == M && out.size(2) == N,
              "gemm_batched: shapes");
  TORCH_CHECK(x.stride(2) == 1 && w.stride(2) == 1 && out.stride(2) == 1, "gemm_batched: unit inner stride");
  TORCH_CHECK(x.stride(0) % 8 == 0 && x.stride(1) % 8 == 0 && w.stride(0) % 8 == 0 && w.stride(1) % 8 == 0 &&
                  out.stride(0) % 8 == 0 && out.stride(1) % 8 == 0,
              "gemm_batched: strides must be multiples of 8 elements");
  c10::cuda::CUDAGuard g(x.device());
  GemmBatchedArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(1);
  a.x_bstride = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(1);
  a.w_bstride = w.stride(0);
  a.c = out.data_ptr();
  a.ldc = out.stride(1);
  a.c_bstride = out.stride(0);
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.batch = (int)B;
  a.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  B200_SP_LAUNCH(gemm_bf16_batched(a, sp_stream()));
}

}  // namespace b200
