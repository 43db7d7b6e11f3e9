// Torch glue of the `_C` extension: argument checks, stream/device guards and
// scratch allocation around the plain launchers of launch.h.
#include <ATen/MemoryOverlap.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "launch.h"
#include "ops.h"

#define B200_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define B200_CHECK_DTYPE(x, t) TORCH_CHECK((x).scalar_type() == (t), #x " has dtype ", (x).scalar_type())
#define B200_LAUNCH(expr)                                                                          \
  do {                                                                                             \
    cudaError_t _e = (expr);                                                                       \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));                      \
  } while (0)

namespace b200 {

static inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

static inline uint32_t* status_ptr(const at::Tensor& status) {
  B200_CHECK_CUDA(status);
  TORCH_CHECK(status.scalar_type() == at::kInt && status.numel() >= 1, "status must be an int32 device word");
  return reinterpret_cast<uint32_t*>(status.data_ptr());
}

void gemm_bf16_out(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                   const at::Tensor& status, int64_t splits) {
  B200_CHECK_CUDA(x);
  B200_CHECK_CUDA(w);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm_bf16: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_bf16: inner dims must be contiguous");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == w.size(0), "gemm_bf16: bad out shape");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat, "gemm_bf16: out bf16 or fp32");
  at::assert_no_partial_overlap(out, x);  // the output must not alias an operand
  at::assert_no_partial_overlap(out, w);
  if (bias.has_value()) {
    B200_CHECK_DTYPE(*bias, at::kBFloat16);
    TORCH_CHECK(bias->numel() == w.size(0) && bias->is_contiguous(), "gemm_bf16: bad bias");
  }
  c10::cuda::CUDAGuard g(x.device());
  GemmArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  a.bias = bias.has_value() ? bias->data_ptr() : nullptr;
  a.c = out.data_ptr();
  a.ldc = out.stride(0);
  a.out_f32 = out.scalar_type() == at::kFloat ? 1 : 0;
  a.M = x.size(0);
  a.N = w.size(0);
  a.K = x.size(1);
  a.status = status_ptr(status);
  a.splits = gemm_bf16_splits(a.M, a.N, a.K, (int)splits);
  at::Tensor partial;
  if (gemm_bf16_uses_partial(a.M, a.splits)) {
    partial = at::empty({(int64_t)a.splits * a.M * a.N}, x.options().dtype(at::kFloat));
    a.partial = partial.data_ptr<float>();
    a.partial_cap = partial.numel();
  }
  B200_LAUNCH(gemm_bf16(a, cur_stream()));
}

void rms_norm_out(at::Tensor& out, const at::Tensor& x, const at::Tensor& w, double eps) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  B200_CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1 && w.is_contiguous(), "rms_norm: layout");
  TORCH_CHECK(out.sizes() == x.sizes() && w.numel() == x.size(1), "rms_norm: shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(rms_norm(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), w.data_ptr(), x.size(0), x.size(1),
                       (float)eps, cur_stream()));
}

void silu_mul_op(at::Tensor& out, const at::Tensor& x, double limit) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && out.dim() == 2 && x.size(1) == 2 * out.size(1) && x.size(0) == out.size(0) &&
                  x.stride(1) == 1 && out.stride(1) == 1,
              "silu_mul: x [T, 2I], out [T, I]");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(silu_mul(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), x.size(0), out.size(1), (float)limit,
                       cur_stream()));
}

void fused_add_rms_norm_(at::Tensor& x, at::Tensor& residual, const at::Tensor& w, double eps) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(residual, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.sizes() == residual.sizes() && x.stride(1) == 1 && residual.stride(1) == 1,
              "fused_add_rms_norm: layout");
  TORCH_CHECK(w.numel() == x.size(1) && w.is_contiguous(), "fused_add_rms_norm: weight");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(fused_add_rms_norm(x.data_ptr(), x.stride(0), residual.data_ptr(), residual.stride(0), w.data_ptr(),
                                 x.size(0), x.size(1), (float)eps, cur_stream()));
}

}  // namespace b200

namespace b200 {

static inline const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

void moe_topk_op(const at::Tensor& logits, int64_t k, int64_t mode, const c10::optional<at::Tensor>& bias,
                 double scale, bool renorm, at::Tensor& ids, at::Tensor& weights) {
  B200_CHECK_CUDA(logits);
  B200_CHECK_DTYPE(logits, at::kFloat);
  TORCH_CHECK(logits.dim() == 2 && logits.is_contiguous(), "moe_topk: logits [T, E] contiguous fp32");
  B200_CHECK_DTYPE(ids, at::kInt);
  B200_CHECK_DTYPE(weights, at::kFloat);
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(ids.numel() == (int64_t)T * k && weights.numel() == (int64_t)T * k, "moe_topk: output size");
  if (bias.has_value()) {
    B200_CHECK_DTYPE(*bias, at::kFloat);
    TORCH_CHECK(bias->numel() == E, "moe_topk: bias size");
  }
  c10::cuda::CUDAGuard g(logits.device());
  B200_LAUNCH(moe_topk(logits.data_ptr<float>(), T, E, (int)k, (int)mode,
                       bias.has_value() ? bias->data_ptr<float>() : nullptr, (float)scale, renorm ? 1 : 0,
                       ids.data_ptr<int>(), weights.data_ptr<float>(), cur_stream()));
}

void moe_build_assignments_op(const at::Tensor& ids, const at::Tensor& weights,
                              const c10::optional<at::Tensor>& expert_map, int64_t E_local, int64_t tile_rows,
                              at::Tensor& sorted_token, at::Tensor& sorted_weight, at::Tensor& slot_of,
                              at::Tensor& items, at::Tensor& num_items, at::Tensor& expert_offsets) {
  B200_CHECK_CUDA(ids);
  B200_CHECK_DTYPE(ids, at::kInt);
  B200_CHECK_DTYPE(weights, at::kFloat);
  TORCH_CHECK(ids.dim() == 2 && ids.is_contiguous() && weights.sizes() == ids.sizes(), "build: ids [T, k]");
  const int T = ids.size(0), k = ids.size(1);
  TORCH_CHECK(sorted_token.numel() >= (int64_t)T * k && sorted_weight.numel() >= (int64_t)T * k &&
                  slot_of.numel() >= (int64_t)T * k,
              "build: assignment buffers too small");
  TORCH_CHECK(items.scalar_type() == at::kInt && items.dim() == 2 && items.size(1) == 4, "build: items [n, 4] int32");
  TORCH_CHECK(expert_offsets.numel() >= E_local + 1, "build: expert_offsets too small");
  c10::cuda::CUDAGuard g(ids.device());
  B200_LAUNCH(moe_build_assignments(
      ids.data_ptr<int>(), weights.data_ptr<float>(), T, k,
      expert_map.has_value() ? expert_map->data_ptr<int>() : nullptr,
      expert_map.has_value() ? (int)expert_map->numel() : (int)E_local, (int)E_local, (int)tile_rows,
      sorted_token.data_ptr<int>(), sorted_weight.data_ptr<float>(), slot_of.data_ptr<int>(),
      reinterpret_cast<int4*>(items.data_ptr<int>()), num_items.data_ptr<int>(), expert_offsets.data_ptr<int>(),
      (int)items.size(0), cur_stream()));
}

void exl3_input_rotate_op(const at::Tensor& x, int64_t in_features, const c10::optional<at::Tensor>& sorted_token,
                          const c10::optional<at::Tensor>& expert_offsets, int64_t E_local, const at::Tensor& suh0,
                          const c10::optional<at::Tensor>& suh1, at::Tensor& out0,
                          const c10::optional<at::Tensor>& out1, int64_t rows,
                          const c10::optional<at::Tensor>& sum0, const c10::optional<at::Tensor>& sum1) {
  B200_CHECK_CUDA(x);
  TORCH_CHECK((!sum0.has_value() || (sum0->scalar_type() == at::kFloat && sum0->numel() >= rows)) &&
                  (!sum1.has_value() || (sum1->scalar_type() == at::kFloat && sum1->numel() >= rows)),
              "rotate: row sums fp32 [rows]");
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(suh0, at::kHalf);
  B200_CHECK_DTYPE(out0, at::kHalf);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "rotate: x rows contiguous");
  const int K = out0.size(-1);
  TORCH_CHECK(suh0.size(-1) == K && out0.is_contiguous() && out0.size(0) >= rows, "rotate: geometry");
  TORCH_CHECK(suh1.has_value() == out1.has_value(), "rotate: suh1/out1 go together");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(exl3_input_rotate(x.data_ptr(), x.stride(0), (int)in_features, K,
                                sorted_token.has_value() ? sorted_token->data_ptr<int>() : nullptr,
                                expert_offsets.has_value() ? expert_offsets->data_ptr<int>() : nullptr, (int)E_local,
                                suh0.data_ptr(), opt_ptr(suh1), suh0.dim() == 2 ? suh0.stride(0) : 0, out0.data_ptr(),
                                out1.has_value() ? out1->data_ptr() : nullptr,
                                sum0.has_value() ? sum0->data_ptr<float>() : nullptr,
                                sum1.has_value() ? sum1->data_ptr<float>() : nullptr, (int)rows, cur_stream()));
}

void exl3_gemm_op(int64_t nmat, const at::Tensor& trellis0, const c10::optional<at::Tensor>& trellis1,
                  const at::Tensor& svh0, const c10::optional<at::Tensor>& svh1,
                  const c10::optional<at::Tensor>& suh_next, int64_t bits_x2, int64_t codebook, const at::Tensor& b0,
                  const c10::optional<at::Tensor>& b1, int64_t tile_rows, const at::Tensor& items,
                  const at::Tensor& num_items, int64_t max_work, at::Tensor& out, int64_t out_mode,
                  double swiglu_limit, const at::Tensor& status, const c10::optional<at::Tensor>& sx0,
                  const c10::optional<at::Tensor>& sx1, int64_t sx_parts, const c10::optional<at::Tensor>& hsum) {
  B200_CHECK_CUDA(trellis0);
  TORCH_CHECK((!sx0.has_value() || sx0->scalar_type() == at::kFloat) &&
                  (!sx1.has_value() || sx1->scalar_type() == at::kFloat) &&
                  (!hsum.has_value() || hsum->scalar_type() == at::kFloat),
              "exl3_gemm: row sums fp32");
  TORCH_CHECK(trellis0.scalar_type() == at::kShort && trellis0.dim() == 4 && trellis0.is_contiguous(),
              "exl3_gemm: trellis [E, K/16, N/16, 8*bits_x2] int16");
  TORCH_CHECK(trellis0.size(3) == 8 * bits_x2, "exl3_gemm: trellis stride vs bits_x2");
  const int K = trellis0.size(1) * 16, N = trellis0.size(2) * 16;
  TORCH_CHECK(nmat == 1 || nmat == 2, "exl3_gemm: nmat");
  if (nmat == 2) {
    TORCH_CHECK(trellis1.has_value() && svh1.has_value() && suh_next.has_value() && b1.has_value(),
                "exl3_gemm: gate/up pass needs both matrices, suh_next and b1");
    TORCH_CHECK(trellis1->sizes() == trellis0.sizes() && trellis1->is_contiguous(), "exl3_gemm: trellis1");
    TORCH_CHECK(out.scalar_type() == at::kHalf, "exl3_gemm: gate/up output is fp16");
  }
  B200_CHECK_DTYPE(svh0, at::kHalf);
  B200_CHECK_DTYPE(b0, at::kHalf);
  TORCH_CHECK(svh0.size(-1) == N && b0.size(-1) == K && b0.is_contiguous(), "exl3_gemm: svh/b geometry");
  TORCH_CHECK(out.stride(-1) == 1 && out.size(-1) >= N, "exl3_gemm: out");
  TORCH_CHECK((out_mode == 0 && out.scalar_type() == at::kHalf) || (out_mode == 1 && out.scalar_type() == at::kFloat) ||
                  (out_mode == 2 && out.scalar_type() == at::kBFloat16),
              "exl3_gemm: out dtype vs out_mode");
  c10::cuda::CUDAGuard g(b0.device());
  Exl3GemmArgs a{};
  a.nmat = (int)nmat;
  a.trellis[0] = trellis0.data_ptr();
  a.trellis[1] = nmat == 2 ? trellis1->data_ptr() : nullptr;
  a.trellis_estride = trellis0.stride(0);
  a.num_experts = trellis0.size(0);
  a.svh[0] = svh0.data_ptr();
  a.svh[1] = nmat == 2 ? svh1->data_ptr() : nullptr;
  a.svh_estride = svh0.dim() == 2 ? svh0.stride(0) : 0;
  a.suh_next = opt_ptr(suh_next);
  a.suh_next_estride = (suh_next.has_value() && suh_next->dim() == 2) ? suh_next->stride(0) : 0;
  a.K = K;
  a.N = N;
  a.bits_x2 = (int)bits_x2;
  a.codebook = (int)codebook;
  a.b0 = b0.data_ptr();
  a.b1 = opt_ptr(b1);
  a.b_rows = b0.size(0);
  a.tile_rows = (int)tile_rows;
  a.items = items.data_ptr<int>();
  a.num_items = num_items.data_ptr<int>();
  a.max_work = (int)max_work;
  a.out = out.data_ptr();
  a.ld_out = out.stride(0);
  a.out_mode = (int)out_mode;
  a.swiglu_limit = (float)swiglu_limit;
  a.sx0 = sx0.has_value() ? sx0->data_ptr<float>() : nullptr;
  a.sx1 = sx1.has_value() ? sx1->data_ptr<float>() : nullptr;
  a.sx_parts = (int)sx_parts;
  a.hsum = hsum.has_value() ? hsum->data_ptr<float>() : nullptr;
  a.status = status_ptr(status);
  B200_LAUNCH(exl3_gemm(a, cur_stream()));
}

void moe_combine_op(const at::Tensor& y, const at::Tensor& slot_of, const at::Tensor& sorted_weight, int64_t k,
                    const c10::optional<at::Tensor>& add, at::Tensor& out) {
  B200_CHECK_CUDA(y);
  B200_CHECK_DTYPE(y, at::kFloat);
  TORCH_CHECK(y.stride(-1) == 1 && out.stride(-1) == 1, "combine: layout");
  const int T = out.size(0), H = out.size(1);
  TORCH_CHECK(slot_of.numel() >= (int64_t)T * k, "combine: slot_of");
  if (add.has_value()) TORCH_CHECK(add->sizes() == out.sizes() && add->stride(0) == out.stride(0), "combine: add");
  c10::cuda::CUDAGuard g(y.device());
  const bool f32 = out.scalar_type() == at::kFloat;
  B200_LAUNCH(moe_combine(y.data_ptr<float>(), y.stride(0), slot_of.data_ptr<int>(), sorted_weight.data_ptr<float>(),
                          T, (int)k, H, opt_ptr(add), f32 ? nullptr : out.data_ptr(), out.stride(0),
                          f32 ? out.data_ptr<float>() : nullptr, cur_stream()));
}

}  // namespace b200

namespace b200 {

void kda_forward_op(const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& state_idx,
                    const c10::optional<at::Tensor>& has_init, const at::Tensor& qkv, const at::Tensor& g_raw,
                    const at::Tensor& beta_raw, const c10::optional<at::Tensor>& g2, at::Tensor& conv_state,
                    const c10::optional<at::Tensor>& conv_w, const c10::optional<at::Tensor>& conv_b,
                    const at::Tensor& a_log, const c10::optional<at::Tensor>& g_bias, double lower_bound,
                    const c10::optional<at::Tensor>& norm_w, double eps, double l2_eps, double q_scale, bool l2norm,
                    at::Tensor& state, at::Tensor& out, const c10::optional<at::Tensor>& verify,
                    const c10::optional<at::Tensor>& rec, int64_t chunk_min_len,
                    const c10::optional<at::Tensor>& chunk_scratch, const c10::optional<at::Tensor>& status,
                    int64_t gate_mode) {
  B200_CHECK_CUDA(qkv);
  B200_CHECK_DTYPE(qkv, at::kBFloat16);
  B200_CHECK_DTYPE(state, at::kFloat);
  B200_CHECK_DTYPE(a_log, at::kFloat);
  TORCH_CHECK(state.dim() == 4 && state.size(2) == 128 && state.size(3) == 128 && state.is_contiguous(),
              "kda: state [slots, H, 128, 128] fp32");
  const int H = state.size(1);
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(1) >= 3 * H * 128 && qkv.stride(1) == 1, "kda: qkv [T, 3*H*128]");
  TORCH_CHECK(g_raw.stride(-1) == 1 && beta_raw.stride(-1) == 1 && out.stride(-1) == 1, "kda: inner strides");
  TORCH_CHECK(conv_state.is_contiguous() && conv_state.size(1) == 3 * H * 128 && conv_state.size(2) == 3,
              "kda: conv_state [slots, 3*H*128, 3]");
  TORCH_CHECK(a_log.numel() == H, "kda: a_log [H]");
  TORCH_CHECK(gate_mode == 0 || gate_mode == 1, "kda: gate_mode 0 (KDA) or 1 (gated delta net)");
  const int64_t gate_width = gate_mode ? H : H * 128;  // per channel (KDA) or per head (gated delta net)
  TORCH_CHECK(g_raw.size(-1) >= gate_width, "kda: g_raw [T, H*128] (KDA) or [T, H] (gated delta net)");
  if (g_bias.has_value())
    TORCH_CHECK(g_bias->scalar_type() == at::kFloat && g_bias->numel() == gate_width, "kda: g_bias");
  TORCH_CHECK(gate_mode == 0 || chunk_min_len == 0, "kda: the chunked prefill takes KDA gates only");
  c10::cuda::CUDAGuard g(qkv.device());
  KdaArgs a{};
  a.full = 1;
  a.H = H;
  a.D = 128;
  a.num_seqs = cu_seqlens.numel() - 1;
  a.cu_seqlens = cu_seqlens.data_ptr<int>();
  a.state_idx = state_idx.has_value() ? state_idx->data_ptr<int>() : nullptr;
  a.has_init = has_init.has_value() ? has_init->data_ptr<int>() : nullptr;
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ld_qkv = qkv.stride(0);
  a.g_raw = reinterpret_cast<const __nv_bfloat16*>(g_raw.data_ptr());
  a.ld_g = g_raw.stride(0);
  a.beta_raw = reinterpret_cast<const __nv_bfloat16*>(beta_raw.data_ptr());
  a.ld_beta = beta_raw.stride(0);
  a.g2 = g2.has_value() ? reinterpret_cast<const __nv_bfloat16*>(g2->data_ptr()) : nullptr;
  a.ld_g2 = g2.has_value() ? g2->stride(0) : 0;
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.conv_w = conv_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(conv_w->data_ptr()) : nullptr;
  a.conv_b = conv_b.has_value() ? reinterpret_cast<const __nv_bfloat16*>(conv_b->data_ptr()) : nullptr;
  a.a_log = a_log.data_ptr<float>();
  a.g_bias = g_bias.has_value() ? g_bias->data_ptr<float>() : nullptr;
  a.lower_bound = (float)lower_bound;
  a.gate_mode = (int)gate_mode;
  a.norm_w = norm_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr()) : nullptr;
  a.eps = (float)eps;
  a.l2_eps = (float)l2_eps;
  a.q_scale = (float)q_scale;
  a.l2norm = l2norm ? 1 : 0;
  a.state = state.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = out.stride(0);
  if (verify.has_value()) {
    TORCH_CHECK(rec.has_value() && rec->scalar_type() == at::kFloat && rec->is_contiguous() &&
                    rec->numel() >= qkv.size(0) * H * 3 * 128 && verify->scalar_type() == at::kInt,
                "kda verify: int32 flags [num_seqs] and fp32 records [T, H, 3, 128]");
    a.verify = verify->data_ptr<int>();
    a.rec = rec->data_ptr<float>();
  }
  if (chunk_min_len > 0) {
    // sequences of at least chunk_min_len tokens in chunks of 64 on the tensor cores, the rest (and
    // everything under speculative verify) through the recurrence
    TORCH_CHECK(!verify.has_value(), "kda: chunked prefill does not record verify updates");
    TORCH_CHECK(chunk_scratch.has_value() && chunk_scratch->is_cuda() && chunk_scratch->is_contiguous() &&
                    (size_t)chunk_scratch->nbytes() >= kda_chunk_scratch_bytes((int)qkv.size(0), H),
                "kda: chunk scratch of kda_chunk_scratch_bytes(T, H) bytes");
    TORCH_CHECK(out.stride(0) >= H * 128 && out.stride(0) % 8 == 0 &&
                    reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
                "kda: chunked output rows must be 16-byte aligned");
    TORCH_CHECK(!g2.has_value() || (g2->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(g2->data_ptr()) % 16 == 0),
                "kda: chunked output gate rows must be 16-byte aligned");
    TORCH_CHECK(!norm_w.has_value() || (norm_w->is_contiguous() &&
                                        reinterpret_cast<uintptr_t>(norm_w->data_ptr()) % 16 == 0),
                "kda: chunked norm weight must be contiguous and 16-byte aligned");
    TORCH_CHECK(status.has_value() && status->scalar_type() == at::kInt, "kda: status word");
    a.skip_long = (int)chunk_min_len;
    B200_LAUNCH(kda_recurrent(a, cur_stream()));
    KdaChunkArgs c{};
    c.k = a;
    c.k.skip_long = 0;
    c.T = (int)qkv.size(0);
    c.min_len = (int)chunk_min_len;
    c.scratch = chunk_scratch->data_ptr();
    c.scratch_bytes = chunk_scratch->nbytes();
    c.status = reinterpret_cast<uint32_t*>(status->data_ptr<int>());
    B200_LAUNCH(kda_chunked(c, cur_stream()));
    return;
  }
  B200_LAUNCH(kda_recurrent(a, cur_stream()));
}

void kda_core_op(const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& state_idx,
                 const c10::optional<at::Tensor>& has_init, const at::Tensor& q, const at::Tensor& k,
                 const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta, at::Tensor& state, at::Tensor& out) {
  B200_CHECK_CUDA(q);
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k, &v, &g, &out}) {
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 3 && t->size(2) == 128,
                "kda_core: fp32 [T, H, 128] contiguous");
  }
  TORCH_CHECK(beta.scalar_type() == at::kFloat && beta.is_contiguous(), "kda_core: beta fp32 [T, H]");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 4, "kda_core: state");
  c10::cuda::CUDAGuard gd(q.device());
  KdaArgs a{};
  a.full = 0;
  a.H = q.size(1);
  a.D = 128;
  a.num_seqs = cu_seqlens.numel() - 1;
  a.cu_seqlens = cu_seqlens.data_ptr<int>();
  a.state_idx = state_idx.has_value() ? state_idx->data_ptr<int>() : nullptr;
  a.has_init = has_init.has_value() ? has_init->data_ptr<int>() : nullptr;
  a.q_f32 = q.data_ptr<float>();
  a.k_f32 = k.data_ptr<float>();
  a.v_f32 = v.data_ptr<float>();
  a.g_f32 = g.data_ptr<float>();
  a.beta_f32 = beta.data_ptr<float>();
  a.q_scale = 1.f;
  a.state = state.data_ptr<float>();
  a.out_f32 = out.data_ptr<float>();
  B200_LAUNCH(kda_recurrent(a, cur_stream()));
}

}  // namespace b200

namespace b200 {

void rope_op(at::Tensor& x, const at::Tensor& positions, const at::Tensor& cos_sin, int64_t offset, int64_t rot_dim,
             bool interleaved, const c10::optional<at::Tensor>& out, int64_t out_offset) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "rope: x [T, heads, dim] with contiguous dim");
  TORCH_CHECK(positions.scalar_type() == at::kInt && cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == rot_dim,
              "rope: positions int32, cos_sin fp32 [max_pos, rot_dim]");
  TORCH_CHECK(offset + rot_dim <= x.size(2) && rot_dim % 2 == 0, "rope: range");
  c10::cuda::CUDAGuard g(x.device());
  if (out.has_value()) {
    TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->dim() == 3 && out->stride(2) == 1 &&
                    out->size(0) == x.size(0) && out->size(1) == x.size(1) && out_offset + rot_dim <= out->size(2),
                "rope: out [T, heads, >= out_offset + rot_dim]");
  }
  B200_LAUNCH(rope_apply(x.data_ptr(), x.stride(0), x.stride(1), x.size(1), (int)offset, (int)rot_dim,
                         positions.data_ptr<int>(), cos_sin.data_ptr<float>(), interleaved ? 1 : 0, x.size(0),
                         cur_stream(), out.has_value() ? out->data_ptr() : nullptr,
                         out.has_value() ? out->stride(0) : 0, out.has_value() ? out->stride(1) : 0, (int)out_offset));
}

void mla_latent_cache_write_op(const at::Tensor& kv, const at::Tensor& norm_w, double eps, const at::Tensor& positions,
                               const at::Tensor& cos_sin, bool interleaved, const at::Tensor& slots, at::Tensor& cache) {
  B200_CHECK_CUDA(kv);
  B200_CHECK_DTYPE(kv, at::kBFloat16);
  B200_CHECK_DTYPE(cache, at::kBFloat16);
  TORCH_CHECK(kv.dim() == 2 && kv.size(1) >= 576 && kv.stride(1) == 1, "latent write: kv [T, 576]");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 576, "latent write: cache [..., 576]");
  TORCH_CHECK(slots.scalar_type() == at::kLong && cos_sin.size(1) == 64, "latent write: slots int64, rope 64");
  c10::cuda::CUDAGuard g(kv.device());
  B200_LAUNCH(mla_latent_cache_write(kv.data_ptr(), kv.stride(0), norm_w.data_ptr(), (float)eps,
                                     positions.data_ptr<int>(), cos_sin.data_ptr<float>(), interleaved ? 1 : 0,
                                     slots.data_ptr<int64_t>(), cache.data_ptr(), kv.size(0), cur_stream()));
}

void mla_index_k_write_op(const at::Tensor& k, const c10::optional<at::Tensor>& ln_w,
                          const c10::optional<at::Tensor>& ln_b, double eps, const at::Tensor& positions,
                          const at::Tensor& cos_sin, bool interleaved, const at::Tensor& slots, at::Tensor& cache,
                          at::Tensor& cache_scale) {
  B200_CHECK_CUDA(k);
  B200_CHECK_DTYPE(k, at::kBFloat16);
  TORCH_CHECK(k.dim() == 2 && k.size(1) == 128 && k.stride(1) == 1, "index k: [T, 128]");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 128 && cache.element_size() == 1, "index k: cache uint8");
  TORCH_CHECK(cache_scale.scalar_type() == at::kFloat, "index k: scale fp32");
  c10::cuda::CUDAGuard g(k.device());
  B200_LAUNCH(mla_index_k_write(k.data_ptr(), k.stride(0), opt_ptr(ln_w), opt_ptr(ln_b), (float)eps,
                                positions.data_ptr<int>(), cos_sin.data_ptr<float>(), cos_sin.size(1),
                                interleaved ? 1 : 0, slots.data_ptr<int64_t>(), cache.data_ptr(),
                                cache_scale.data_ptr<float>(), k.size(0), cur_stream()));
}

void mla_index_q_prep_op(const at::Tensor& q, const at::Tensor& positions, const at::Tensor& cos_sin, bool interleaved,
                         const at::Tensor& w, double wscale, at::Tensor& q8, at::Tensor& w_out) {
  B200_CHECK_CUDA(q);
  B200_CHECK_DTYPE(q, at::kBFloat16);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.stride(2) == 1 && q.stride(1) == 128, "index q: [T, H, 128]");
  TORCH_CHECK(q8.is_contiguous() && q8.numel() == q.size(0) * q.size(1) * 128 && q8.element_size() == 1, "index q8");
  TORCH_CHECK(w_out.scalar_type() == at::kFloat && w_out.numel() == q.size(0) * q.size(1), "index w_out");
  B200_CHECK_DTYPE(w, at::kBFloat16);
  c10::cuda::CUDAGuard g(q.device());
  B200_LAUNCH(mla_index_q_prep(q.data_ptr(), q.stride(0), q.size(1), positions.data_ptr<int>(),
                               cos_sin.data_ptr<float>(), cos_sin.size(1), interleaved ? 1 : 0, w.data_ptr(),
                               w.stride(0), (float)wscale, q8.data_ptr(), w_out.data_ptr<float>(), q.size(0),
                               cur_stream()));
}

void mla_indexer_scores_op(const at::Tensor& q8, const at::Tensor& w, const at::Tensor& k_cache,
                           const at::Tensor& k_scale, const at::Tensor& ctx_lens, const c10::optional<at::Tensor>& token_seq,
                           const at::Tensor& block_table, int64_t max_ctx, at::Tensor& scores, const at::Tensor& status) {
  B200_CHECK_CUDA(q8);
  TORCH_CHECK(q8.element_size() == 1 && q8.is_contiguous() && q8.size(-1) == 128 && q8.size(-2) == 64,
              "indexer: q8 [T, 64, 128] fp8");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "indexer: w fp32 [T, 64]");
  TORCH_CHECK(k_cache.element_size() == 1 && k_cache.is_contiguous() && k_cache.size(-1) == 128, "indexer: cache");
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.stride(1) == 1 && scores.size(1) >= max_ctx,
              "indexer: scores [T, >= max_ctx] fp32");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2, "indexer: block_table int32 [S, n]");
  c10::cuda::CUDAGuard g(q8.device());
  const int T = q8.size(0);
  TORCH_CHECK(scores.size(0) >= T && ctx_lens.numel() >= T && w.numel() >= (int64_t)T * 64 &&
                  (!token_seq.has_value() || token_seq->numel() >= T),
              "indexer: scores / ctx_lens / token_seq / w must cover the ", T, " tokens of q8");
  B200_LAUNCH(mla_indexer_scores(q8.data_ptr(), w.data_ptr<float>(), T, k_cache.data_ptr(), k_cache.numel() / 128,
                                 k_scale.data_ptr<float>(), ctx_lens.data_ptr<int>(),
                                 token_seq.has_value() ? token_seq->data_ptr<int>() : nullptr,
                                 block_table.data_ptr<int>(), block_table.stride(0), scores.data_ptr<float>(),
                                 scores.stride(0), (int)max_ctx, status_ptr(status), cur_stream()));
}

void mla_topk_op(const at::Tensor& scores, const at::Tensor& ctx_lens, int64_t k,
                 const c10::optional<at::Tensor>& token_seq, const at::Tensor& block_table, int64_t block_size,
                 at::Tensor& out_idx, at::Tensor& out_count) {
  B200_CHECK_CUDA(scores);
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.stride(1) == 1, "topk: scores fp32");
  TORCH_CHECK(out_idx.scalar_type() == at::kInt && out_idx.is_contiguous() && out_idx.size(1) == k, "topk: out");
  // the tokens are out_idx's rows; the scores buffer may hold more rows (a graph's shared buffer)
  const int64_t T = out_idx.size(0);
  TORCH_CHECK(scores.size(0) >= T && ctx_lens.numel() >= T && out_count.numel() >= T &&
                  (!token_seq.has_value() || token_seq->numel() >= T),
              "topk: scores / ctx_lens / token_seq / out_count must cover the ", T, " tokens of out_idx");
  TORCH_CHECK(ctx_lens.scalar_type() == at::kInt && out_count.scalar_type() == at::kInt, "topk: int32 lengths");
  c10::cuda::CUDAGuard g(scores.device());
  B200_LAUNCH(mla_topk(scores.data_ptr<float>(), scores.stride(0), ctx_lens.data_ptr<int>(), (int)k,
                       token_seq.has_value() ? token_seq->data_ptr<int>() : nullptr, block_table.data_ptr<int>(),
                       block_table.stride(0), (int)block_size, out_idx.data_ptr<int>(), out_count.data_ptr<int>(),
                       (int)T, cur_stream()));
}

void mla_sparse_attention_op(const at::Tensor& q, const at::Tensor& cache, const at::Tensor& indices,
                             const at::Tensor& counts, double sm_scale, int64_t splits, at::Tensor& out,
                             const c10::optional<at::Tensor>& lse, const at::Tensor& status,
                             const c10::optional<at::Tensor>& sink, int64_t only_half) {
  TORCH_CHECK(only_half >= -1 && only_half <= 1, "sparse attn: only_half -1 (both), 0 or 1");
  TORCH_CHECK(only_half < 0 || !lse.has_value(), "sparse attn: the log-sum-exp comes with both halves");
  B200_CHECK_CUDA(q);
  B200_CHECK_DTYPE(q, at::kBFloat16);
  TORCH_CHECK(q.dim() == 3 && (q.size(2) == 576 || q.size(2) == 512) && q.is_contiguous(),
              "sparse attn: q [T, nh, 576 or 512] contiguous");
  const int dim = (int)q.size(2);
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.is_contiguous() && cache.size(-1) == dim,
              "sparse attn: cache rows must match q's width");
  if (sink.has_value())
    TORCH_CHECK(sink->scalar_type() == at::kFloat && sink->is_cuda() && sink->is_contiguous() &&
                    sink->numel() == q.size(1),
                "sparse attn: sink fp32 [nh]");
  TORCH_CHECK(indices.scalar_type() == at::kInt && indices.is_contiguous() && indices.size(0) == q.size(0),
              "sparse attn: indices [T, topk] int32");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(-1) == 512 &&
                  out.numel() >= q.size(0) * q.size(1) * 512,
              "sparse attn: out [T, nh, 512]");
  TORCH_CHECK(counts.scalar_type() == at::kInt && counts.numel() >= q.size(0), "sparse attn: counts int32 [T]");
  c10::cuda::CUDAGuard g(q.device());
  const int T = q.size(0), nh = q.size(1);
  at::Tensor part_o, part_ml;
  if (splits > 1) {
    part_o = at::empty({splits, T, nh, 512}, q.options().dtype(at::kFloat));
    part_ml = at::empty({splits, T, nh, 2}, q.options().dtype(at::kFloat));
  }
  B200_LAUNCH(mla_sparse_attention(q.data_ptr(), T, nh, dim, cache.data_ptr(), indices.data_ptr<int>(),
                                   counts.data_ptr<int>(), indices.size(1), (float)sm_scale, (int)splits,
                                   out.data_ptr(), splits > 1 ? part_o.data_ptr<float>() : nullptr,
                                   splits > 1 ? part_ml.data_ptr<float>() : nullptr,
                                   lse.has_value() ? lse->data_ptr<float>() : nullptr,
                                   sink.has_value() ? sink->data_ptr<float>() : nullptr, status_ptr(status),
                                   cur_stream(), (int)only_half));
}

}  // namespace b200

namespace b200 {

void sample_rows_op(const at::Tensor& logits, const c10::optional<at::Tensor>& temperature, int64_t seed,
                    const c10::optional<at::Tensor>& step, int64_t vocab_offset, at::Tensor& out_val,
                    at::Tensor& out_idx, const c10::optional<at::Tensor>& bans) {
  B200_CHECK_CUDA(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample: logits [rows, V]");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "sample: bf16/fp32");
  TORCH_CHECK(out_val.scalar_type() == at::kFloat && out_idx.scalar_type() == at::kInt, "sample: outputs");
  if (temperature.has_value()) TORCH_CHECK(temperature->scalar_type() == at::kFloat, "sample: temperature fp32");
  if (step.has_value()) TORCH_CHECK(step->scalar_type() == at::kLong, "sample: step int64");
  if (temperature.has_value()) TORCH_CHECK(temperature->numel() >= logits.size(0), "sample: temperature rows");
  if (bans.has_value())
    TORCH_CHECK(bans->scalar_type() == at::kInt && bans->dim() == 2 && bans->is_contiguous() &&
                    bans->size(0) >= logits.size(0) && bans->size(1) <= 4,
                "sample: bans [rows, <= 4] int32 contiguous");
  TORCH_CHECK(out_val.numel() >= logits.size(0) && out_idx.numel() >= logits.size(0), "sample: output rows");
  c10::cuda::CUDAGuard g(logits.device());
  B200_LAUNCH(sample_rows(logits.data_ptr(), logits.scalar_type() == at::kFloat ? 1 : 0, logits.stride(0),
                          logits.size(0), logits.size(1),
                          temperature.has_value() ? temperature->data_ptr<float>() : nullptr, (uint64_t)seed,
                          step.has_value() ? step->data_ptr<int64_t>() : nullptr, (int)vocab_offset,
                          bans.has_value() ? bans->data_ptr<int>() : nullptr,
                          bans.has_value() ? (int)bans->size(1) : 0, out_val.data_ptr<float>(),
                          out_idx.data_ptr<int>(), cur_stream()));
}

void sample_combine_op(const at::Tensor& vals, const at::Tensor& idx, at::Tensor& out) {
  B200_CHECK_CUDA(vals);
  TORCH_CHECK(vals.dim() == 2 && idx.sizes() == vals.sizes() && out.scalar_type() == at::kLong, "combine: shapes");
  c10::cuda::CUDAGuard g(vals.device());
  B200_LAUNCH(sample_combine(vals.data_ptr<float>(), idx.data_ptr<int>(), vals.size(0), vals.size(1),
                             out.data_ptr<int64_t>(), cur_stream()));
}

}  // namespace b200

namespace b200 {

void symm_all_reduce_op(const at::Tensor& in, at::Tensor& out, const at::Tensor& peers, int64_t rank, int64_t world,
                        int64_t data_off, int64_t half_bytes, at::Tensor& epochs, const at::Tensor& status,
                        double timeout_s) {
  B200_CHECK_CUDA(in);
  B200_CHECK_DTYPE(in, at::kBFloat16);
  TORCH_CHECK(in.is_contiguous() && out.is_contiguous() && out.sizes() == in.sizes(), "symm_all_reduce: layout");
  TORCH_CHECK(in.numel() % 8 == 0, "symm_all_reduce: element count must be a multiple of 8");
  TORCH_CHECK(peers.scalar_type() == at::kLong && peers.numel() == world && peers.is_cuda(), "symm_all_reduce: peers");
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.is_cuda(), "symm_all_reduce: epochs int32");
  c10::cuda::CUDAGuard g(in.device());
  B200_LAUNCH(symm_all_reduce(in.data_ptr(), out.data_ptr(), in.numel(),
                              reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), (int)rank, (int)world,
                              data_off, half_bytes, reinterpret_cast<uint32_t*>(epochs.data_ptr<int>()),
                              (int)epochs.numel(), status_ptr(status), (uint64_t)(timeout_s * 1e9), cur_stream()));
}

}  // namespace b200

namespace b200 {

void dequant_gemm_op(int64_t format, int64_t nmat, const at::Tensor& w0, const c10::optional<at::Tensor>& w1,
                     const at::Tensor& s0, const c10::optional<at::Tensor>& s1, const at::Tensor& b0,
                     const c10::optional<at::Tensor>& b1, int64_t tile_rows, const at::Tensor& items,
                     const at::Tensor& num_items, int64_t max_work, at::Tensor& out, int64_t out_mode,
                     double swiglu_limit, const at::Tensor& status) {
  B200_CHECK_CUDA(w0);
  TORCH_CHECK(w0.dim() == 3 && w0.is_contiguous(), "dequant_gemm: weights [E, ...] contiguous");
  DequantGemmArgs a{};
  a.format = (int)format;
  a.nmat = (int)nmat;
  a.E = w0.size(0);
  if (format == 0) {
    TORCH_CHECK(w0.scalar_type() == at::kInt, "marlin: packed int32 [E, K/16, 2N]");
    a.K = w0.size(1) * 16;
    a.N = w0.size(2) / 2;
    TORCH_CHECK(s0.scalar_type() == at::kBFloat16 && s0.size(1) == a.K / 128 && s0.size(2) == a.N, "marlin scales");
  } else {
    TORCH_CHECK(w0.element_size() == 1, "fp8: weights [E, N, K] one byte each");
    a.N = w0.size(1);
    a.K = w0.size(2);
    TORCH_CHECK(s0.scalar_type() == at::kFloat && s0.size(1) == a.N / 128 && s0.size(2) == a.K / 128, "fp8 scales");
  }
  TORCH_CHECK(s0.is_contiguous(), "dequant_gemm: scales contiguous");
  if (nmat == 2) {
    TORCH_CHECK(w1.has_value() && s1.has_value() && b1.has_value(), "dequant_gemm: gate/up needs w1, s1, b1");
    TORCH_CHECK(w1->sizes() == w0.sizes() && w1->is_contiguous(), "dequant_gemm: w1 shape");
  }
  TORCH_CHECK(b0.is_contiguous() && b0.size(-1) == a.K, "dequant_gemm: activations [rows, K]");
  TORCH_CHECK(b0.scalar_type() == (format == 0 ? at::kBFloat16 : at::kHalf), "dequant_gemm: activation dtype");
  c10::cuda::CUDAGuard g(b0.device());
  a.w[0] = w0.data_ptr();
  a.w[1] = nmat == 2 ? w1->data_ptr() : nullptr;
  a.scale[0] = s0.data_ptr();
  a.scale[1] = nmat == 2 ? s1->data_ptr() : nullptr;
  a.b0 = b0.data_ptr();
  a.b1 = opt_ptr(b1);
  a.b_rows = b0.size(0);
  a.tile_rows = (int)tile_rows;
  a.items = items.data_ptr<int>();
  a.num_items = num_items.data_ptr<int>();
  a.max_work = (int)max_work;
  a.out = out.data_ptr();
  a.ld_out = out.stride(0);
  a.out_mode = (int)out_mode;
  a.swiglu_limit = (float)swiglu_limit;
  a.status = status_ptr(status);
  B200_LAUNCH(dequant_gemm(a, cur_stream()));
}

void gather_rows_op(const at::Tensor& x, const c10::optional<at::Tensor>& src, at::Tensor& out, int64_t rows) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.is_contiguous() && out.size(-1) == x.size(1), "gather_rows");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kHalf, "gather_rows: out bf16/fp16");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(gather_rows(x.data_ptr(), x.stride(0), x.size(1), src.has_value() ? src->data_ptr<int>() : nullptr,
                          out.data_ptr(), out.scalar_type() == at::kHalf ? 1 : 0, (int)rows, cur_stream()));
}

}  // namespace b200

namespace b200 {

void gemm_allreduce_op(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                       const at::Tensor& peers, int64_t rank, int64_t world, int64_t flag_off, int64_t data_off,
                       int64_t tile_bytes_cap, int64_t max_ctas, at::Tensor& epochs, const at::Tensor& status,
                       double timeout_s) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  B200_CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm_allreduce: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_allreduce: inner dims contiguous");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == w.size(0), "gemm_allreduce: bad out shape");
  TORCH_CHECK(peers.scalar_type() == at::kLong && peers.numel() == world && peers.is_cuda(), "gemm_allreduce: peers");
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= max_ctas, "gemm_allreduce: epochs");
  if (bias.has_value()) {
    B200_CHECK_DTYPE(*bias, at::kBFloat16);
    TORCH_CHECK(bias->numel() == w.size(0) && bias->is_contiguous(), "gemm_allreduce: bad bias");
  }
  c10::cuda::CUDAGuard g(x.device());
  GemmArArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  a.bias = bias.has_value() ? bias->data_ptr() : nullptr;
  a.c = out.data_ptr();
  a.ldc = out.stride(0);
  a.M = x.size(0);
  a.N = w.size(0);
  a.K = x.size(1);
  a.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.rank = (int)rank;
  a.world = (int)world;
  a.flag_off = flag_off;
  a.data_off = data_off;
  a.tile_bytes_cap = tile_bytes_cap;
  a.max_ctas = (int)max_ctas;
  a.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr<int>());
  a.status = status_ptr(status);
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  B200_LAUNCH(gemm_bf16_allreduce(a, cur_stream()));
}

void combine_allreduce_op(const at::Tensor& y, const at::Tensor& slot_of, const at::Tensor& sorted_weight, int64_t k,
                          const c10::optional<at::Tensor>& add, at::Tensor& out, const at::Tensor& peers,
                          int64_t rank, int64_t world, int64_t flag_off, int64_t data_off, int64_t slot_bytes,
                          at::Tensor& epochs, const at::Tensor& status, double timeout_s) {
  B200_CHECK_CUDA(y);
  B200_CHECK_DTYPE(y, at::kFloat);
  B200_CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(y.stride(1) == 1 && out.is_contiguous() && out.dim() == 2, "combine_allreduce: layout");
  TORCH_CHECK(slot_of.scalar_type() == at::kInt && slot_of.is_contiguous(), "combine_allreduce: slot_of int32");
  TORCH_CHECK(sorted_weight.scalar_type() == at::kFloat, "combine_allreduce: weights fp32");
  if (add.has_value()) {
    B200_CHECK_DTYPE(*add, at::kBFloat16);
    TORCH_CHECK(add->is_contiguous() && add->sizes() == out.sizes(), "combine_allreduce: add");
  }
  c10::cuda::CUDAGuard g(y.device());
  CombineArArgs a{};
  a.y = y.data_ptr<float>();
  a.ld_y = y.stride(0);
  a.slot_of = slot_of.data_ptr<int>();
  a.sorted_weight = sorted_weight.data_ptr<float>();
  a.k = (int)k;
  a.add = add.has_value() ? reinterpret_cast<const __nv_bfloat16*>(add->data_ptr()) : nullptr;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.T = out.size(0);
  a.H = out.size(1);
  a.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.rank = (int)rank;
  a.world = (int)world;
  a.flag_off = flag_off;
  a.data_off = data_off;
  a.slot_bytes = slot_bytes;
  a.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr<int>());
  a.status = status_ptr(status);
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  B200_LAUNCH(combine_allreduce(a, (int)epochs.numel(), cur_stream()));
}

}  // namespace b200

namespace b200 {

void timing_stamp_op(at::Tensor& ring, const at::Tensor& cursor, int64_t col) {
  B200_CHECK_CUDA(ring);
  TORCH_CHECK(ring.scalar_type() == at::kLong && ring.dim() == 2 && ring.is_contiguous(), "timing ring int64 [rows, w]");
  TORCH_CHECK(cursor.scalar_type() == at::kInt && cursor.is_cuda(), "timing cursor int32");
  c10::cuda::CUDAGuard g(ring.device());
  B200_LAUNCH(timing_stamp(ring.data_ptr<int64_t>(), cursor.data_ptr<int>(), (int)ring.size(1), (int)col,
                           cur_stream()));
}

void timing_open_row_op(at::Tensor& ring, at::Tensor& cursor, at::Tensor& step_counter) {
  B200_CHECK_CUDA(ring);
  TORCH_CHECK(ring.scalar_type() == at::kLong && ring.dim() == 2 && ring.is_contiguous(), "timing ring int64 [rows, w]");
  TORCH_CHECK(step_counter.scalar_type() == at::kLong && step_counter.is_cuda(), "timing step counter int64");
  c10::cuda::CUDAGuard g(ring.device());
  B200_LAUNCH(timing_open_row(ring.data_ptr<int64_t>(), cursor.data_ptr<int>(), (int)ring.size(0), (int)ring.size(1),
                              step_counter.data_ptr<int64_t>(), cur_stream()));
}

}  // namespace b200

namespace b200 {

void dequant_rows_op(const at::Tensor& rows, int64_t D, const c10::optional<at::Tensor>& failed, at::Tensor& out) {
  B200_CHECK_CUDA(rows);
  TORCH_CHECK(rows.scalar_type() == at::kByte && rows.dim() == 2 && rows.is_contiguous(), "rows: uint8 [n, row_bytes]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == rows.size(0) &&
                  out.size(1) == D,
              "out: bf16 [n, D]");
  if (failed.has_value())
    TORCH_CHECK(failed->scalar_type() == at::kByte && failed->is_cuda() && failed->numel() == rows.size(0),
                "failed: device uint8 [n]");
  c10::cuda::CUDAGuard g(rows.device());
  B200_LAUNCH(dequant_rows_e4m3(rows.data_ptr(), rows.size(1), (int)D,
                                failed.has_value() ? failed->data_ptr<uint8_t>() : nullptr, out.data_ptr(),
                                (int)rows.size(0), cur_stream()));
}

void ple_decode_op(const at::Tensor& rows, const at::Tensor& ids, const at::Tensor& head_bias,
                   const at::Tensor& head_offsets, const at::Tensor& head_vocab, int64_t owner_lo, int64_t owner_hi,
                   int64_t bits, const c10::optional<at::Tensor>& failed, at::Tensor& out) {
  B200_CHECK_CUDA(rows);
  TORCH_CHECK(rows.scalar_type() == at::kShort && rows.dim() == 2 && rows.is_contiguous(),
              "ple_decode: rows int16 [n, 1 + dim*bits/16]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.is_contiguous() &&
                  out.size(0) == rows.size(0),
              "ple_decode: out bf16 [n, dim]");
  const int64_t n = rows.size(0), dim = out.size(1), heads = head_bias.size(0);
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_cuda() && ids.is_contiguous() && ids.numel() == n,
              "ple_decode: ids device int64 [n]");
  TORCH_CHECK(head_bias.scalar_type() == at::kHalf && head_bias.is_cuda() && head_bias.is_contiguous() &&
                  head_bias.dim() == 2 && head_bias.size(1) == dim && heads > 0,
              "ple_decode: head_bias fp16 [heads, dim]");
  for (const at::Tensor* t : {&head_offsets, &head_vocab})
    TORCH_CHECK(t->scalar_type() == at::kLong && t->is_cuda() && t->is_contiguous() && t->numel() == heads,
                "ple_decode: head offsets / vocab sizes device int64 [heads]");
  TORCH_CHECK(bits >= 1 && bits <= 16 && (dim * bits) % 16 == 0 && rows.size(1) == 1 + dim * bits / 16,
              "ple_decode: rows must be [n, 1 + dim*bits/16] with bits in [1, 16] and dim*bits a multiple of 16");
  TORCH_CHECK(0 <= owner_lo && owner_lo <= owner_hi, "ple_decode: owner range");
  if (failed.has_value())
    TORCH_CHECK(failed->scalar_type() == at::kByte && failed->is_cuda() && failed->numel() == n,
                "ple_decode: failed device uint8 [n]");
  c10::cuda::CUDAGuard g(rows.device());
  B200_LAUNCH(ple_decode_rows(rows.data_ptr(), rows.size(1), ids.data_ptr<int64_t>(), head_bias.data_ptr(),
                              head_offsets.data_ptr<int64_t>(), head_vocab.data_ptr<int64_t>(), (int)heads, (int)dim,
                              (int)bits, owner_lo, owner_hi,
                              failed.has_value() ? failed->data_ptr<uint8_t>() : nullptr, out.data_ptr(), (int)n,
                              cur_stream()));
}

}  // namespace b200

namespace b200 {

void kda_recover_op(const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& state_idx, const at::Tensor& keep,
                    const at::Tensor& rec, at::Tensor& state, const at::Tensor& qkv,
                    const c10::optional<at::Tensor>& conv_state) {
  B200_CHECK_CUDA(rec);
  TORCH_CHECK(rec.scalar_type() == at::kFloat && state.scalar_type() == at::kFloat && keep.scalar_type() == at::kInt,
              "kda_recover: fp32 records/state, int32 keep");
  c10::cuda::CUDAGuard g(rec.device());
  KdaRecoverArgs a{};
  a.H = state.size(1);
  a.num_seqs = cu_seqlens.numel() - 1;
  a.cu_seqlens = cu_seqlens.data_ptr<int>();
  a.state_idx = state_idx.has_value() ? state_idx->data_ptr<int>() : nullptr;
  a.keep = keep.data_ptr<int>();
  a.rec = rec.data_ptr<float>();
  a.state = state.data_ptr<float>();
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ld_qkv = qkv.stride(0);
  a.conv_state = conv_state.has_value() ? reinterpret_cast<__nv_bfloat16*>(conv_state->data_ptr()) : nullptr;
  B200_LAUNCH(kda_recover(a, cur_stream()));
}

void mhc_post_pre_op(const c10::optional<at::Tensor>& x, const at::Tensor& H, const c10::optional<at::Tensor>& post,
                     const c10::optional<at::Tensor>& comb, const at::Tensor& fn, const at::Tensor& scale,
                     const at::Tensor& base, const at::Tensor& norm_w, const c10::optional<at::Tensor>& pre_mix,
                     double rms_eps, double eps, double post_mult, int64_t iters, double norm_eps, int64_t mode,
                     at::Tensor& H_out, at::Tensor& y, at::Tensor& post_out, at::Tensor& comb_out, at::Tensor& pre_out) {
  B200_CHECK_CUDA(H);
  TORCH_CHECK(H.dim() == 3 && H.is_contiguous() && H.scalar_type() == at::kBFloat16, "mhc: H [T, hc, d] bf16");
  const int64_t T = H.size(0), hc = H.size(1), d = H.size(2);
  const int64_t N = 2 * hc + hc * hc;
  TORCH_CHECK(fn.scalar_type() == at::kFloat && fn.is_contiguous() && fn.size(0) == N && fn.size(1) == hc * d,
              "mhc: fn [2 hc + hc^2, hc d] fp32");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() >= 3 && base.scalar_type() == at::kFloat &&
                  base.numel() == N && norm_w.scalar_type() == at::kBFloat16 && norm_w.numel() == d,
              "mhc: scale [3] / base [N] fp32, norm_w [d] bf16");
  TORCH_CHECK(H_out.is_contiguous() && H_out.sizes() == H.sizes() && y.is_contiguous() && y.size(0) == T &&
                  y.size(1) == d && post_out.is_contiguous() && comb_out.is_contiguous() && pre_out.is_contiguous(),
              "mhc: output shapes");
  if (x.has_value()) {
    TORCH_CHECK(x->is_contiguous() && x->scalar_type() == at::kBFloat16 && x->size(0) == T && x->size(1) == d &&
                    post.has_value() && comb.has_value() && post->is_contiguous() && comb->is_contiguous() &&
                    post->scalar_type() == at::kFloat && comb->scalar_type() == at::kFloat,
                "mhc: x [T, d] bf16 with post [T, hc] / comb [T, hc, hc] fp32");
  }
  TORCH_CHECK(mode != 1 || (pre_mix.has_value() && pre_mix->is_contiguous() && pre_mix->scalar_type() == at::kFloat),
              "mhc: mode 1 needs pre_mix [T, hc] fp32");
  c10::cuda::CUDAGuard g(H.device());
  MhcArgs a{};
  a.x = x.has_value() ? reinterpret_cast<const __nv_bfloat16*>(x->data_ptr()) : nullptr;
  a.H = reinterpret_cast<const __nv_bfloat16*>(H.data_ptr());
  a.post = post.has_value() ? post->data_ptr<float>() : nullptr;
  a.comb = comb.has_value() ? comb->data_ptr<float>() : nullptr;
  a.fn = fn.data_ptr<float>();
  a.scale = scale.data_ptr<float>();
  a.base = base.data_ptr<float>();
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  a.pre_mix = pre_mix.has_value() ? pre_mix->data_ptr<float>() : nullptr;
  a.rms_eps = (float)rms_eps;
  a.eps = (float)eps;
  a.post_mult = (float)post_mult;
  a.norm_eps = (float)norm_eps;
  a.iters = (int)iters;
  a.mode = (int)mode;
  a.T = (int)T;
  a.hc = (int)hc;
  a.d = (int)d;
  a.H_out = reinterpret_cast<__nv_bfloat16*>(H_out.data_ptr());
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.post_out = post_out.data_ptr<float>();
  a.comb_out = comb_out.data_ptr<float>();
  a.pre_out = pre_out.data_ptr<float>();
  B200_LAUNCH(mhc_post_pre(a, cur_stream()));
}

}  // namespace b200

namespace b200 {

// Gated grouped-query attention (gqa.cu + the dense mode of the block attention kernel).
void gqa_prep_op(const at::Tensor& proj, int64_t nh, int64_t nkv, const at::Tensor& q_norm_w,
                 const at::Tensor& k_norm_w, double eps, const at::Tensor& positions, const at::Tensor& cos_sin,
                 const at::Tensor& slots, at::Tensor& q_out, at::Tensor& cache) {
  B200_CHECK_CUDA(proj);
  B200_CHECK_DTYPE(proj, at::kBFloat16);
  TORCH_CHECK(proj.dim() == 2 && proj.stride(1) == 1 && proj.size(1) >= nh * 512 + nkv * 512,
              "gqa prep: proj [T, nh*512 + nkv*512]");
  TORCH_CHECK(nkv >= 1 && nh % nkv == 0, "gqa prep: query heads must be a multiple of key-value heads");
  const int T = proj.size(0);
  TORCH_CHECK(q_norm_w.scalar_type() == at::kBFloat16 && q_norm_w.numel() == 256 && q_norm_w.is_contiguous() &&
                  k_norm_w.scalar_type() == at::kBFloat16 && k_norm_w.numel() == 256 && k_norm_w.is_contiguous(),
              "gqa prep: q / k norm weights bf16 [256]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.numel() >= T, "gqa prep: positions int32 [T]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.dim() == 2,
              "gqa prep: cos_sin fp32 [max_pos, rot_dim]");
  TORCH_CHECK(slots.scalar_type() == at::kLong && slots.numel() >= T, "gqa prep: slots int64 [T]");
  TORCH_CHECK(q_out.scalar_type() == at::kBFloat16 && q_out.is_contiguous() && q_out.numel() >= (int64_t)T * nh * 512,
              "gqa prep: q_out [T * nkv, group, 512]");
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.is_contiguous() && cache.size(-1) == 512,
              "gqa prep: cache rows [.., 512]");
  c10::cuda::CUDAGuard g(proj.device());
  GqaPrepArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ld_proj = proj.stride(0);
  a.nh = (int)nh;
  a.nkv = (int)nkv;
  a.group = (int)(nh / nkv);
  a.q_norm_w = reinterpret_cast<const __nv_bfloat16*>(q_norm_w.data_ptr());
  a.k_norm_w = reinterpret_cast<const __nv_bfloat16*>(k_norm_w.data_ptr());
  a.eps = (float)eps;
  a.positions = positions.data_ptr<int>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.rot_dim = (int)cos_sin.size(1);
  a.slots = slots.data_ptr<int64_t>();
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  a.cache = reinterpret_cast<__nv_bfloat16*>(cache.data_ptr());
  B200_LAUNCH(gqa_prep(a, T, cur_stream()));
}

void gqa_attention_op(const at::Tensor& q, const at::Tensor& cache, const at::Tensor& ctx_lens,
                      const at::Tensor& token_seq, const at::Tensor& block_table, int64_t kv_heads, double sm_scale,
                      int64_t splits, at::Tensor& out, const at::Tensor& status) {
  B200_CHECK_CUDA(q);
  B200_CHECK_DTYPE(q, at::kBFloat16);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 512 && q.is_contiguous() && q.size(0) % kv_heads == 0,
              "gqa attention: q [T * kv_heads, group, 512] contiguous");
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.is_contiguous() && cache.size(-1) == 512,
              "gqa attention: cache rows [.., 512]");
  const int Tq = q.size(0), group = q.size(1);
  const int T = Tq / kv_heads;
  TORCH_CHECK(ctx_lens.scalar_type() == at::kInt && ctx_lens.numel() >= T && token_seq.scalar_type() == at::kInt &&
                  token_seq.numel() >= T,
              "gqa attention: ctx_lens / token_seq int32 [T]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 && block_table.stride(1) == 1,
              "gqa attention: block_table int32 [S, max_blocks]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() >= (int64_t)Tq * group * 512,
              "gqa attention: out [T * kv_heads, group, 512]");
  TORCH_CHECK(splits >= 1, "gqa attention: splits >= 1");
  at::assert_no_partial_overlap(out, q);
  at::assert_no_partial_overlap(out, cache);
  c10::cuda::CUDAGuard g(q.device());
  at::Tensor part_o, part_ml;
  if (splits > 1) {
    part_o = at::empty({splits, Tq, group, 512}, q.options().dtype(at::kFloat));
    part_ml = at::empty({splits, Tq, group, 2}, q.options().dtype(at::kFloat));
  }
  B200_LAUNCH(gqa_dense_attention(q.data_ptr(), Tq, group, cache.data_ptr(), ctx_lens.data_ptr<int>(),
                                  token_seq.data_ptr<int>(), block_table.data_ptr<int>(), block_table.stride(0),
                                  (int)kv_heads, (float)sm_scale, (int)splits, out.data_ptr(),
                                  splits > 1 ? part_o.data_ptr<float>() : nullptr,
                                  splits > 1 ? part_ml.data_ptr<float>() : nullptr, status_ptr(status), cur_stream()));
}

void gqa_gate_op(const at::Tensor& attn, const at::Tensor& proj, int64_t nh, at::Tensor& out) {
  B200_CHECK_CUDA(attn);
  TORCH_CHECK(attn.scalar_type() == at::kBFloat16 && attn.is_contiguous() && attn.size(-1) == 512,
              "gqa gate: attention rows [T * nh, 512]");
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.dim() == 2 && proj.stride(1) == 1 &&
                  proj.size(1) >= nh * 512 && reinterpret_cast<uintptr_t>(proj.data_ptr()) % 16 == 0,
              "gqa gate: proj [T, >= nh*512], 16-byte aligned");
  const int T = proj.size(0);
  TORCH_CHECK(attn.numel() >= (int64_t)T * nh * 512, "gqa gate: attention rows cover T * nh");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.stride(1) == 1 && out.size(0) >= T &&
                  out.size(1) >= nh * 256 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "gqa gate: out [T, nh*256], 16-byte aligned");
  at::assert_no_partial_overlap(out, attn);
  at::assert_no_partial_overlap(out, proj);
  c10::cuda::CUDAGuard g(attn.device());
  B200_LAUNCH(gqa_gate(attn.data_ptr(), proj.data_ptr(), proj.stride(0), T, (int)nh, out.data_ptr(), out.stride(0),
                       cur_stream()));
}

}  // namespace b200

namespace b200 {

void engram_gate_op(const at::Tensor& h, const at::Tensor& kv, const at::Tensor& wh, const at::Tensor& wk, double eps,
                    at::Tensor& out) {
  B200_CHECK_CUDA(h);
  const int T = h.size(0), H = h.size(1);
  auto rows_ok = [&](const at::Tensor& x, int64_t width) {
    return x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(0) >= T && x.size(1) >= width &&
           x.stride(1) == 1 && x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0;
  };
  TORCH_CHECK(rows_ok(h, H) && H % 8 == 0, "engram gate: h bf16 [T, H], H a multiple of 8, 16-byte rows");
  TORCH_CHECK(rows_ok(kv, 2 * H), "engram gate: kv bf16 [T, 2H] = [k | v], 16-byte rows");
  TORCH_CHECK(rows_ok(out, H), "engram gate: out bf16 [T, H], 16-byte rows");
  TORCH_CHECK(wh.scalar_type() == at::kBFloat16 && wh.numel() == H && wh.is_contiguous() &&
                  wk.scalar_type() == at::kBFloat16 && wk.numel() == H && wk.is_contiguous(),
              "engram gate: norm weights bf16 [H]");
  at::assert_no_partial_overlap(out, h);
  at::assert_no_partial_overlap(out, kv);
  c10::cuda::CUDAGuard g(h.device());
  B200_LAUNCH(engram_gate(h.data_ptr(), h.stride(0), kv.data_ptr(), kv.stride(0), wh.data_ptr(), wk.data_ptr(),
                          (float)eps, T, H, out.data_ptr(), out.stride(0), cur_stream()));
}

}  // namespace b200

namespace b200 {

void dsv4_index_scores_op(const at::Tensor& q, const at::Tensor& w, const at::Tensor& keys,
                          const at::Tensor& block_table, const at::Tensor& seq, const at::Tensor& n_vis,
                          int64_t heads_per_group, at::Tensor& scores) {
  B200_CHECK_CUDA(q);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(),
              "dsv4 index scores: q bf16 [T, H, 128] contiguous");
  const int T = q.size(0), H = q.size(1);
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.numel() >= (int64_t)T * H,
              "dsv4 index scores: w bf16 [T, H]");
  TORCH_CHECK(keys.scalar_type() == at::kBFloat16 && keys.is_contiguous() && keys.size(-1) == 128,
              "dsv4 index scores: keys bf16 [rows, 128]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 && block_table.stride(1) == 1,
              "dsv4 index scores: block_table int32 [S, blocks]");
  TORCH_CHECK(seq.scalar_type() == at::kInt && seq.numel() >= T && n_vis.scalar_type() == at::kInt &&
                  n_vis.numel() >= T,
              "dsv4 index scores: seq / n_vis int32 [T]");
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.dim() == 2 && scores.size(0) >= T &&
                  scores.stride(1) == 1,
              "dsv4 index scores: scores fp32 [T, N]");
  TORCH_CHECK(heads_per_group >= 1 && H % heads_per_group == 0, "dsv4 index scores: rank groups divide the heads");
  c10::cuda::CUDAGuard g(q.device());
  B200_LAUNCH(dsv4_index_scores(q.data_ptr(), w.data_ptr(), keys.data_ptr(), block_table.data_ptr<int>(),
                                block_table.stride(0), seq.data_ptr<int>(), n_vis.data_ptr<int>(), T, H,
                                (int)heads_per_group, scores.data_ptr<float>(), scores.stride(0),
                                (int)scores.size(1), cur_stream()));
}

}  // namespace b200

namespace b200 {

void dsv4_rot_qdq_op(const at::Tensor& x, at::Tensor& out, const at::Tensor& positions, int64_t heads,
                     const at::Tensor& freqs, bool inverse, const c10::optional<at::Tensor>& norm_w, double eps,
                     int64_t mode) {
  B200_CHECK_CUDA(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "dsv4 rot: x bf16 [rows, D]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.stride(1) == 1 &&
                  out.sizes() == x.sizes(),
              "dsv4 rot: out bf16 like x");
  const int rows = x.size(0), D = x.size(1);
  TORCH_CHECK(heads >= 1 && positions.scalar_type() == at::kLong && positions.numel() * heads >= rows,
              "dsv4 rot: positions int64 [rows / heads]");
  TORCH_CHECK(freqs.scalar_type() == at::kFloat && freqs.is_contiguous() && 2 * freqs.numel() <= D,
              "dsv4 rot: freqs fp32 [pairs]");
  if (norm_w.has_value())
    TORCH_CHECK(norm_w->scalar_type() == at::kBFloat16 && norm_w->numel() == D && norm_w->is_contiguous(),
                "dsv4 rot: norm weight bf16 [D]");
  TORCH_CHECK(D % 32 == 0 && D <= 512 && mode >= 0 && mode <= 3, "dsv4 rot: D a multiple of 32 up to 512, mode 0-3");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(dsv4_rot_qdq(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), rows, D,
                           positions.data_ptr<int64_t>(), (int)heads, freqs.data_ptr<float>(), (int)freqs.numel(),
                           inverse ? 1 : 0, norm_w.has_value() ? norm_w->data_ptr() : nullptr, (float)eps, (int)mode,
                           cur_stream()));
}

}  // namespace b200
