// KDA (gated delta rule, per-channel decay) recurrence: decode steps,
// speculative verify and prefill in one kernel.
//
// Reference semantics: vllm_sm80/models/glm5next/ops/kda_decode.py:1-60
// (`kda_decode_v2`: causal conv1d + SiLU on q/k/v, L2 norm, decay gate
// exp(lb * sigmoid(exp(A_log) * (g + bias))), the recurrence
// S <- S*e; u = (v - S k) * beta; S += u k^T; o = S q, and the gated RMSNorm
// with sigmoid(g2)), oracle tests/kernels/test_ampere_pp_kda_prefill.py:228-248.
//
// The gated delta net of the Qwen3-Next-style linear-attention layers is the same recurrence with one
// decay per head, exp(-exp(A_log) * softplus(a + dt_bias)), and a SiLU output gate (gate_mode 1).
//
// B200 layout: one CTA per (sequence, head), 16 warps; warp w owns value rows
// 8w..8w+7 as two groups of four.  Lane = (row-in-group rs: 2 bits, column
// group cg: 3 bits); a thread holds 16 key columns {32j + 4cg + i} of its row
// in each group (32 fp32 state registers).  A row reduction over the 128 key
// columns is 15 in-thread adds and 3 shuffles.  The per-token vectors (q, k,
// decay, v) go through shared memory once; two CTA barriers per token.
// The state is read once and written once per call (tokens of a sequence are
// processed in order inside the kernel), so a decode step is bound by the
// 2 x 64 KiB state traffic per (sequence, head).
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace kda {

constexpr int D = 128;
constexpr int kThreads = 512;

struct ItemIn {
  float x;       // pre-conv q/k/v channel value, or the gate pre-activation, of the first token
  float cw[4];   // conv taps of the channel
  float cb;      // conv bias
  float win[3];  // conv window (zeros for a fresh sequence)
  float beta;    // beta pre-activation (gate thread 0)
  float g2;      // output gate pre-activation of the column (threads < D)
  float nw;      // output norm weight of the column (threads < D)
  float a_h;     // exp(A_log) of the head
};

template <bool FULL>
__global__ void __launch_bounds__(kThreads, 1) kda_recurrent_kernel(KdaArgs p) {
  pdl_prologue();
  // Persistent: CTA c runs the (sequence, head) items c, c + grid, ...  An item's 64 KiB state is
  // bulk-copied into one half of a shared double buffer and moved into registers at the item's
  // start; the half is then free, so the copy of the item two ahead is issued into it at once and
  // two state copies are in flight while the item computes.  Each item's final state is written
  // straight from registers, so state reads and writes stream at the rate of the memory system
  // instead of one load -> compute -> store per CTA.
  extern __shared__ __align__(128) float sbuf[];  // [2][D * D]
  __shared__ __align__(8) uint64_t fullb[2];
  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int rs = lane >> 3, cg = lane & 7;
  const int HD = p.H * D;
  const int items = p.num_seqs * p.H;

  __shared__ __align__(16) float raw_s[3][D];  // q, k, v of the current token (post conv+silu)
  __shared__ __align__(16) float e_s[D];
  __shared__ __align__(16) float o_s[D];
  __shared__ float beta_s;

  // sequences of at least skip_long tokens belong to the chunked kernel: no tokens, no state traffic here
  auto skipped_of = [&](int seq) {
    return p.skip_long > 0 && p.cu_seqlens[seq + 1] - p.cu_seqlens[seq] >= p.skip_long;
  };
  auto has_init_of = [&](int seq) { return p.has_init ? (p.has_init[seq] != 0) : true; };
  // issue the state copy of `item` into buffer `b` (an empty transaction when it has no state)
  auto prefetch = [&](int item, int b) {
    const int sq = item / p.H, hh = item % p.H;
    const int sl = p.state_idx ? p.state_idx[sq] : sq;
    if (has_init_of(sq) && !skipped_of(sq)) {
      mbar_arrive_expect_tx(&fullb[b], D * D * 4);
      bulk_load(sbuf + b * D * D, p.state + ((int64_t)sl * p.H + hh) * D * D, D * D * 4, &fullb[b]);
    } else {
      mbar_arrive_expect_tx(&fullb[b], 0);
    }
  };
  if (tid == 0) {
    mbar_init(&fullb[0], 1);
    mbar_init(&fullb[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0 && (int)blockIdx.x < items) prefetch(blockIdx.x, 0);
  if (tid == 0 && (int)(blockIdx.x + gridDim.x) < items) prefetch(blockIdx.x + gridDim.x, 1);

  // per-thread inputs of an item's first token (FULL): this thread's pre-conv channel value
  // (q/k/v threads) or gate pre-activation (gate threads), its conv taps and window, beta, the
  // output gate and norm weight of its column -- everything the item reads from global memory
  // the sequence metadata of an item (token range, state slot, fresh flag), read one item ahead
  // so that the input loads below do not wait on it
  struct Meta {
    int tt, tend, sl, init;
  };
  auto load_meta = [&](int it) {
    const int sq = it / p.H;
    return Meta{p.cu_seqlens[sq], skipped_of(sq) ? p.cu_seqlens[sq] : p.cu_seqlens[sq + 1],
                p.state_idx ? p.state_idx[sq] : sq,
                has_init_of(sq) ? 1 : 0};
  };
  auto load_inputs = [&](int it, const Meta& m) {
    ItemIn r{};
    if (!FULL) return r;
    const int hh = it % p.H;
    const int tt = m.tt;
    if (tt == m.tend) return r;
    const int sl = m.sl;
    const int wh = tid / D, cc = tid % D;
    if (tid < 3 * D) {
      const int64_t g = (int64_t)wh * HD + hh * D + cc;
      r.x = __bfloat162float(p.qkv[(int64_t)tt * p.ld_qkv + g]);
      if (p.conv_w) {
#pragma unroll
        for (int i = 0; i < 4; ++i) r.cw[i] = __bfloat162float(p.conv_w[g * 4 + i]);
        if (p.conv_b) r.cb = __bfloat162float(p.conv_b[g]);
        if (m.init) {
          const __nv_bfloat16* cs = p.conv_state + ((int64_t)sl * 3 * HD + g) * 3;
#pragma unroll
          for (int i = 0; i < 3; ++i) r.win[i] = __bfloat162float(cs[i]);
        }
      }
    } else {
      r.x = __bfloat162float(p.g_raw[(int64_t)tt * p.ld_g + (p.gate_mode ? hh : hh * D + (tid - 3 * D))]);
      if (tid == 3 * D) r.beta = __bfloat162float(p.beta_raw[(int64_t)tt * p.ld_beta + hh]);
    }
    if (tid < D) {
      if (p.norm_w) r.nw = __bfloat162float(p.norm_w[tid]);
      if (p.g2) r.g2 = __bfloat162float(p.g2[(int64_t)tt * p.ld_g2 + hh * D + tid]);
    }
    if (p.a_log) r.a_h = __expf(p.a_log[hh]);
    return r;
  };
  ItemIn in = (int)blockIdx.x < items ? load_inputs(blockIdx.x, load_meta(blockIdx.x)) : ItemIn{};

  int local = 0;
  for (int item = blockIdx.x; item < items; item += gridDim.x, ++local) {
  const int seq = item / p.H;
  const int h = item % p.H;
  const bool skipped = skipped_of(seq);
  const int t0 = p.cu_seqlens[seq], t1 = skipped ? t0 : p.cu_seqlens[seq + 1];
  const int slot = p.state_idx ? p.state_idx[seq] : seq;
  const bool has_init = has_init_of(seq) && !skipped;
  const bool verify = p.verify != nullptr && p.verify[seq] != 0 && p.rec != nullptr;
  const int buf = local & 1;
  const bool has_next = item + (int)gridDim.x < items;
  const Meta next_meta = has_next ? load_meta(item + gridDim.x) : Meta{0, 0, 0, 0};
  const bool landed = mbar_wait(&fullb[buf], (local >> 1) & 1, nullptr);

  float* S = p.state + ((int64_t)slot * p.H + h) * D * D;
  const float* Ss = sbuf + buf * D * D;
  float st[2][4][4];
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    const int row = warp * 8 + gi * 4 + rs;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 v = (has_init && landed) ? *reinterpret_cast<const float4*>(Ss + row * D + j * 32 + cg * 4)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
      st[gi][j][0] = v.x;
      st[gi][j][1] = v.y;
      st[gi][j][2] = v.z;
      st[gi][j][3] = v.w;
    }
  }
  __syncthreads();  // every thread has its state in registers: the buffer is free
  if (tid == 0 && item + 2 * (int)gridDim.x < items) {
    fence_proxy_async_smem();  // the generic-proxy reads above before the async-proxy refill
    prefetch(item + 2 * gridDim.x, buf);
  }

  // conv window of this thread's channel (FULL mode, threads 0..383); the item's first-token
  // inputs arrived in `in` (loaded while the previous item computed)
  const int which = tid / D, c = tid % D;
  const int64_t gc = (int64_t)which * HD + h * D + c;  // channel in the [q | k | v] layout
  ItemIn cur = in;
  float win[3] = {cur.win[0], cur.win[1], cur.win[2]};
  const float qscale = p.q_scale;

  for (int t = t0; t < t1; ++t) {
    const bool first = t == t0;
    // ---------------------------------------------------------------- (a) token vectors
    if (tid < 3 * D) {
      float x;
      if (FULL) {
        x = first ? cur.x : __bfloat162float(p.qkv[(int64_t)t * p.ld_qkv + gc]);
        if (p.conv_w) {
          float y = cur.cb + cur.cw[0] * win[0] + cur.cw[1] * win[1] + cur.cw[2] * win[2] + cur.cw[3] * x;
          win[0] = win[1];
          win[1] = win[2];
          win[2] = x;
          x = __bfloat162float(__float2bfloat16(siluf_(y)));
        }
      } else {
        const float* src = which == 0 ? p.q_f32 : which == 1 ? p.k_f32 : p.v_f32;
        x = src[((int64_t)t * p.H + h) * D + c];
      }
      raw_s[which][c] = x;
    } else {
      const int cc = tid - 3 * D;  // 0..127
      float e;
      if (FULL) {
        const int gi = p.gate_mode ? h : h * D + cc;
        const float g = (first ? cur.x : __bfloat162float(p.g_raw[(int64_t)t * p.ld_g + gi])) +
                        (p.g_bias ? p.g_bias[gi] : 0.f);
        e = p.gate_mode ? __expf(-cur.a_h * softplusf_(g)) : __expf(p.lower_bound * sigmoidf_(cur.a_h * g));
      } else {
        e = __expf(p.g_f32[((int64_t)t * p.H + h) * D + cc]);
      }
      e_s[cc] = e;
      if (cc == 0) {
        beta_s = FULL ? sigmoidf_(first ? cur.beta : __bfloat162float(p.beta_raw[(int64_t)t * p.ld_beta + h]))
                      : p.beta_f32[(int64_t)t * p.H + h];
      }
    }
    __syncthreads();
    // ---------------------------------------------------------------- (b) norms + recurrence
    float qn = qscale, kn = 1.f;
    if (FULL && p.l2norm) {
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = raw_s[0][lane * 4 + i], b = raw_s[1][lane * 4 + i];
        sq += a * a;
        sk += b * b;
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      qn = qscale * rsqrtf(sq + p.l2_eps);
      kn = rsqrtf(sk + p.l2_eps);
    }
    const float beta = beta_s;
    if (verify && tid < D) {  // the token's normalised key and decay (what the recurrence applies)
      float* r = p.rec + ((int64_t)t * p.H + h) * 3 * D;
      r[D + tid] = raw_s[1][tid] * kn;
      r[2 * D + tid] = e_s[tid];
    }
    // decay and S k over the key columns (column blocks j outer: the token vectors are reread from
    // shared memory rather than held, and each row's sums keep their j-then-i order)
    float kv[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 k4 = *reinterpret_cast<const float4*>(&raw_s[1][j * 32 + cg * 4]);
      const float4 e4 = *reinterpret_cast<const float4*>(&e_s[j * 32 + cg * 4]);
      const float kj[4] = {k4.x * kn, k4.y * kn, k4.z * kn, k4.w * kn};
      const float ej[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
      for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          st[gi][j][i] *= ej[i];
          kv[gi] = fmaf(st[gi][j][i], kj[i], kv[gi]);
        }
    }
    float u[2];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int row = warp * 8 + gi * 4 + rs;
      float v = kv[gi];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      u[gi] = (raw_s[2][row] - v) * beta;
      if (verify && cg == 0) p.rec[(((int64_t)t * p.H + h) * 3 + 0) * D + row] = u[gi];
    }
    float o[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 k4 = *reinterpret_cast<const float4*>(&raw_s[1][j * 32 + cg * 4]);
      const float4 q4 = *reinterpret_cast<const float4*>(&raw_s[0][j * 32 + cg * 4]);
      const float kj[4] = {k4.x * kn, k4.y * kn, k4.z * kn, k4.w * kn};
      const float qj[4] = {q4.x * qn, q4.y * qn, q4.z * qn, q4.w * qn};
#pragma unroll
      for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          st[gi][j][i] = fmaf(u[gi], kj[i], st[gi][j][i]);
          o[gi] = fmaf(st[gi][j][i], qj[i], o[gi]);
        }
    }
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int row = warp * 8 + gi * 4 + rs;
      float v = o[gi];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      if (cg == 0) o_s[row] = v;
    }
    // the next item's first-token inputs: in flight during the output and the write-back
    if (t + 1 == t1 && has_next) in = load_inputs(item + gridDim.x, next_meta);
    __syncthreads();
    // ---------------------------------------------------------------- (c) output (gated RMSNorm)
    if (tid < D) {
      const float o = o_s[tid];
      if (FULL && p.norm_w) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = o_s[lane * 4 + i];
          ss += a * a;
        }
        ss = warp_sum(ss);
        float y = o * rsqrtf(ss / D + p.eps) * cur.nw;
        if (p.g2) {
          const float z = first ? cur.g2 : __bfloat162float(p.g2[(int64_t)t * p.ld_g2 + h * D + tid]);
          y *= p.gate_mode ? z * sigmoidf_(z) : sigmoidf_(z);
        }
        p.out[(int64_t)t * p.ld_out + h * D + tid] = __float2bfloat16(y);
      } else if (p.out_f32) {
        p.out_f32[((int64_t)t * p.H + h) * D + tid] = o;
      } else {
        p.out[(int64_t)t * p.ld_out + h * D + tid] = __float2bfloat16(o);
      }
    }
  }
  if (t0 == t1 && has_next) in = load_inputs(item + gridDim.x, next_meta);  // (no token ran)
  // ------------------------------------------------------------------ write back
  if (verify || skipped) continue;  // kda_recover applies the accepted prefix later; or chunked
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    const int row = warp * 8 + gi * 4 + rs;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      *reinterpret_cast<float4*>(S + row * D + j * 32 + cg * 4) =
          make_float4(st[gi][j][0], st[gi][j][1], st[gi][j][2], st[gi][j][3]);
    }
  }
  if (FULL && p.conv_w && tid < 3 * D && t1 > t0) {
    __nv_bfloat16* cs = p.conv_state + ((int64_t)slot * 3 * HD + gc) * 3;
#pragma unroll
    for (int i = 0; i < 3; ++i) cs[i] = __float2bfloat16(win[i]);
  }
  }  // items
}

// S <- S * e_t + u_t k_t^T for the first keep[s] recorded tokens (the same per-element operations,
// in the same order, as the recurrence itself, so the result equals having run only those tokens),
// then the conv window advanced past them.
__global__ void __launch_bounds__(kThreads) kda_recover_kernel(KdaRecoverArgs p) {
  pdl_prologue();
  const int seq = blockIdx.x / p.H;
  const int h = blockIdx.x % p.H;
  const int n = p.keep[seq];
  if (n <= 0) return;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int rs = lane >> 3, cg = lane & 7;
  const int t0 = p.cu_seqlens[seq];
  const int slot = p.state_idx ? p.state_idx[seq] : seq;
  float* S = p.state + ((int64_t)slot * p.H + h) * D * D;
  float st[2][4][4];
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    const int row = warp * 8 + gi * 4 + rs;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(S + row * D + j * 32 + cg * 4);
      st[gi][j][0] = v.x;
      st[gi][j][1] = v.y;
      st[gi][j][2] = v.z;
      st[gi][j][3] = v.w;
    }
  }
  for (int t = t0; t < t0 + n; ++t) {
    const float* r = p.rec + ((int64_t)t * p.H + h) * 3 * D;
    float kk[4][4], ee[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 k4 = *reinterpret_cast<const float4*>(r + D + j * 32 + cg * 4);
      const float4 e4 = *reinterpret_cast<const float4*>(r + 2 * D + j * 32 + cg * 4);
      kk[j][0] = k4.x; kk[j][1] = k4.y; kk[j][2] = k4.z; kk[j][3] = k4.w;
      ee[j][0] = e4.x; ee[j][1] = e4.y; ee[j][2] = e4.z; ee[j][3] = e4.w;
    }
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int row = warp * 8 + gi * 4 + rs;
      const float u = r[row];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) st[gi][j][i] = fmaf(u, kk[j][i], st[gi][j][i] * ee[j][i]);
    }
  }
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    const int row = warp * 8 + gi * 4 + rs;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(S + row * D + j * 32 + cg * 4) =
          make_float4(st[gi][j][0], st[gi][j][1], st[gi][j][2], st[gi][j][3]);
  }
  if (p.conv_state && tid < 3 * D) {
    // window after the kept tokens: the last three pre-conv inputs, older ones from the old window
    const int HD = p.H * D;
    const int which = tid / D, c = tid % D;
    const int64_t gc = (int64_t)which * HD + h * D + c;
    __nv_bfloat16* cs = p.conv_state + ((int64_t)slot * 3 * HD + gc) * 3;
    float w[3] = {__bfloat162float(cs[0]), __bfloat162float(cs[1]), __bfloat162float(cs[2])};
    for (int t = t0; t < t0 + n; ++t) {
      w[0] = w[1];
      w[1] = w[2];
      w[2] = __bfloat162float(p.qkv[(int64_t)t * p.ld_qkv + gc]);
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) cs[i] = __float2bfloat16(w[i]);
  }
}

}  // namespace kda

cudaError_t kda_recover(const KdaRecoverArgs& a, cudaStream_t stream) {
  if (a.num_seqs == 0) return cudaSuccess;
  launch_pdl(kda::kda_recover_kernel, dim3(a.num_seqs * a.H), dim3(kda::kThreads), 0, stream, a);
  return cudaGetLastError();
}

cudaError_t kda_recurrent(const KdaArgs& a, cudaStream_t stream) {
  if (a.num_seqs == 0) return cudaSuccess;
  if (a.D != kda::D) return cudaErrorInvalidValue;
  const int items = a.num_seqs * a.H;
  const int grid = std::min(items, device_sm_count());
  const int smem = 2 * kda::D * kda::D * 4;
  auto kern = a.full ? kda::kda_recurrent_kernel<true> : kda::kda_recurrent_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  launch_pdl(kern, dim3(grid), dim3(kda::kThreads), smem, stream, a);
  return cudaGetLastError();
}

}  // namespace b200
