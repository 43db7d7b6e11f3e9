// KDA (gated delta rule, per-channel decay) recurrence: decode steps,
// speculative verify and prefill in one kernel.
//
// Reference semantics: vllm_sm80/models/glm5next/ops/kda_decode.py:1-60
// (`kda_decode_v2`: causal conv1d + SiLU on q/k/v, L2 norm, decay gate
// exp(lb * sigmoid(exp(A_log) * (g + bias))), the recurrence
// S <- S*e; u = (v - S k) * beta; S += u k^T; o = S q, and the gated RMSNorm
// with sigmoid(g2)), oracle tests/kernels/test_ampere_pp_kda_prefill.py:228-248.
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
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace kda {

constexpr int D = 128;
constexpr int kThreads = 512;

template <bool FULL>
__global__ void __launch_bounds__(kThreads) kda_recurrent_kernel(KdaArgs p) {
  const int seq = blockIdx.x / p.H;
  const int h = blockIdx.x % p.H;
  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int rs = lane >> 3, cg = lane & 7;
  const int t0 = p.cu_seqlens[seq], t1 = p.cu_seqlens[seq + 1];
  const int slot = p.state_idx ? p.state_idx[seq] : seq;
  const bool has_init = p.has_init ? (p.has_init[seq] != 0) : true;
  const bool verify = p.verify != nullptr && p.verify[seq] != 0 && p.rec != nullptr;
  const int HD = p.H * D;

  __shared__ __align__(16) float raw_s[3][D];  // q, k, v of the current token (post conv+silu)
  __shared__ __align__(16) float e_s[D];
  __shared__ __align__(16) float o_s[D];
  __shared__ float beta_s;

  float* S = p.state + ((int64_t)slot * p.H + h) * D * D;
  float st[2][4][4];
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    const int row = warp * 8 + gi * 4 + rs;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 v = has_init ? *reinterpret_cast<const float4*>(S + row * D + j * 32 + cg * 4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      st[gi][j][0] = v.x;
      st[gi][j][1] = v.y;
      st[gi][j][2] = v.z;
      st[gi][j][3] = v.w;
    }
  }

  // conv window of this thread's channel (FULL mode, threads 0..383)
  float win[3] = {0.f, 0.f, 0.f};
  float cw[4] = {0.f, 0.f, 0.f, 0.f};
  float cb = 0.f;
  int which = tid / D, c = tid % D;
  int64_t gc = (int64_t)which * HD + h * D + c;  // channel in the [q | k | v] layout
  if (FULL && tid < 3 * D) {
    if (p.conv_w) {
#pragma unroll
      for (int i = 0; i < 4; ++i) cw[i] = __bfloat162float(p.conv_w[gc * 4 + i]);
      if (p.conv_b) cb = __bfloat162float(p.conv_b[gc]);
      if (has_init) {
        const __nv_bfloat16* cs = p.conv_state + ((int64_t)slot * 3 * HD + gc) * 3;
#pragma unroll
        for (int i = 0; i < 3; ++i) win[i] = __bfloat162float(cs[i]);
      }
    }
  }
  float a_h = 0.f;
  if (FULL && p.a_log) a_h = __expf(p.a_log[h]);
  const float qscale = p.q_scale;

  for (int t = t0; t < t1; ++t) {
    // ---------------------------------------------------------------- (a) token vectors
    if (tid < 3 * D) {
      float x;
      if (FULL) {
        x = __bfloat162float(p.qkv[(int64_t)t * p.ld_qkv + gc]);
        if (p.conv_w) {
          float y = cb + cw[0] * win[0] + cw[1] * win[1] + cw[2] * win[2] + cw[3] * x;
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
        const float g = __bfloat162float(p.g_raw[(int64_t)t * p.ld_g + h * D + cc]) + (p.g_bias ? p.g_bias[h * D + cc] : 0.f);
        e = __expf(p.lower_bound * sigmoidf_(a_h * g));
      } else {
        e = __expf(p.g_f32[((int64_t)t * p.H + h) * D + cc]);
      }
      e_s[cc] = e;
      if (cc == 0) {
        beta_s = FULL ? sigmoidf_(__bfloat162float(p.beta_raw[(int64_t)t * p.ld_beta + h]))
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
    float kk[4][4], qq[4][4], ee[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 k4 = *reinterpret_cast<const float4*>(&raw_s[1][j * 32 + cg * 4]);
      const float4 q4 = *reinterpret_cast<const float4*>(&raw_s[0][j * 32 + cg * 4]);
      const float4 e4 = *reinterpret_cast<const float4*>(&e_s[j * 32 + cg * 4]);
      kk[j][0] = k4.x * kn; kk[j][1] = k4.y * kn; kk[j][2] = k4.z * kn; kk[j][3] = k4.w * kn;
      qq[j][0] = q4.x * qn; qq[j][1] = q4.y * qn; qq[j][2] = q4.z * qn; qq[j][3] = q4.w * qn;
      ee[j][0] = e4.x; ee[j][1] = e4.y; ee[j][2] = e4.z; ee[j][3] = e4.w;
    }
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int row = warp * 8 + gi * 4 + rs;
      float kv = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          st[gi][j][i] *= ee[j][i];
          kv = fmaf(st[gi][j][i], kk[j][i], kv);
        }
      kv += __shfl_xor_sync(0xffffffffu, kv, 1);
      kv += __shfl_xor_sync(0xffffffffu, kv, 2);
      kv += __shfl_xor_sync(0xffffffffu, kv, 4);
      const float u = (raw_s[2][row] - kv) * beta;
      if (verify && cg == 0) p.rec[(((int64_t)t * p.H + h) * 3 + 0) * D + row] = u;
      float o = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          st[gi][j][i] = fmaf(u, kk[j][i], st[gi][j][i]);
          o = fmaf(st[gi][j][i], qq[j][i], o);
        }
      o += __shfl_xor_sync(0xffffffffu, o, 1);
      o += __shfl_xor_sync(0xffffffffu, o, 2);
      o += __shfl_xor_sync(0xffffffffu, o, 4);
      if (cg == 0) o_s[row] = o;
    }
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
        float y = o * rsqrtf(ss / D + p.eps) * __bfloat162float(p.norm_w[tid]);
        if (p.g2) y *= sigmoidf_(__bfloat162float(p.g2[(int64_t)t * p.ld_g2 + h * D + tid]));
        p.out[(int64_t)t * p.ld_out + h * D + tid] = __float2bfloat16(y);
      } else if (p.out_f32) {
        p.out_f32[((int64_t)t * p.H + h) * D + tid] = o;
      } else {
        p.out[(int64_t)t * p.ld_out + h * D + tid] = __float2bfloat16(o);
      }
    }
  }

  // ------------------------------------------------------------------ write back
  if (verify) return;  // kda_recover applies the accepted prefix later
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
}

// S <- S * e_t + u_t k_t^T for the first keep[s] recorded tokens (the same per-element operations,
// in the same order, as the recurrence itself, so the result equals having run only those tokens),
// then the conv window advanced past them.
__global__ void __launch_bounds__(kThreads) kda_recover_kernel(KdaRecoverArgs p) {
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
  kda::kda_recover_kernel<<<a.num_seqs * a.H, kda::kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t kda_recurrent(const KdaArgs& a, cudaStream_t stream) {
  if (a.num_seqs == 0) return cudaSuccess;
  if (a.D != kda::D) return cudaErrorInvalidValue;
  const int grid = a.num_seqs * a.H;
  if (a.full)
    kda::kda_recurrent_kernel<true><<<grid, kda::kThreads, 0, stream>>>(a);
  else
    kda::kda_recurrent_kernel<false><<<grid, kda::kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace b200
