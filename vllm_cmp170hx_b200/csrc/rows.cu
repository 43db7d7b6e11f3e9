// Dequantisation of table rows fetched from storage (the reference's Engram
// E4M3 x E8M0 dequant, models/deepseek_v41/ops/sm80_engram_dequant.py, and
// the NaN poison of failed rows, csrc/exl3/ple.cu:91).
//
// A row of D values is stored as D e4m3 bytes followed by D/32 E8M0 scale
// bytes (value = e4m3 * 2^(e - 127)).  One warp per row: lane l converts 8
// consecutive codes at a time (cvt.rn.f16x2.e4m3x2), applies the block scale
// and writes bf16.  A row flagged failed by the host reader is written as
// NaN, so its tokens fail in the failed-input path instead of running on
// garbage.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace {

__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  const __half2 hh = *reinterpret_cast<__half2*>(&h);
  return __half22float2(hh);
}

__global__ void dequant_rows_kernel(const uint8_t* __restrict__ rows, int64_t row_bytes, int D,
                                    const uint8_t* __restrict__ failed, __nv_bfloat16* __restrict__ out, int n) {
  pdl_prologue();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= n) return;
  const uint8_t* row = rows + (int64_t)warp * row_bytes;
  const uint8_t* scales = row + D;
  __nv_bfloat16* o = out + (int64_t)warp * D;
  const bool bad = failed && failed[warp];
  for (int c = lane * 8; c < D; c += 32 * 8) {
    const uint2 codes = *reinterpret_cast<const uint2*>(row + c);
    const float s = exp2f((float)scales[c / 32] - 127.f);
    const uint16_t* p = reinterpret_cast<const uint16_t*>(&codes);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = e4m3x2_to_float2(p[i]);
      v[2 * i] = f.x * s;
      v[2 * i + 1] = f.y * s;
    }
    uint4 pk;
    if (bad) {
      pk = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);  // bf16 NaN
    } else {
      pk.x = pack_bf16x2(v[0], v[1]);
      pk.y = pack_bf16x2(v[2], v[3]);
      pk.z = pack_bf16x2(v[4], v[5]);
      pk.w = pack_bf16x2(v[6], v[7]);
    }
    *reinterpret_cast<uint4*>(o + c) = pk;
  }
}

}  // namespace

cudaError_t dequant_rows_e4m3(const void* rows, int64_t row_bytes, int D, const uint8_t* failed, void* out, int n,
                              cudaStream_t stream) {
  if (D % 256 != 0 || row_bytes < D + D / 32 || row_bytes % 8 != 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int threads = 256, warps = threads / 32;
  launch_pdl(dequant_rows_kernel, dim3((n + warps - 1) / warps), dim3(threads), 0, stream, 
      reinterpret_cast<const uint8_t*>(rows), row_bytes, D, failed, reinterpret_cast<__nv_bfloat16*>(out), n);
  return cudaGetLastError();
}

}  // namespace b200

namespace b200 {

// ============================================================================
// EXL3-coded per-layer-embedding (PLE) rows (the reference's selected-row
// decoder, csrc/exl3/ple.cu:91, and its format, models/qwen4_exp/exl3_ple.py).
//
// A packed row is 1 + dim*bits/16 16-bit words: an fp16 row scale, then a
// tail-biting ring of dim*bits bits (bit i in word i/16 at position i%16),
// channel c owning ring bits [c*bits, (c+1)*bits).  Channel c's 16-bit
// trellis state takes its own bits as the low field and the fields of
// channels c-1, c-2, ... (mod dim) above them.  The state goes through the
// EXL3 "mul1" codebook (state * 0x83DCD12D, the four product bytes summed,
// fp16(1024 + sum) * a + b rounded once to fp16), then the row scale (fp32
// product, exact) and the head's fp16 bias (fp32 add) and rounds to bf16.
//
// Ids outside [owner_lo, owner_hi) (another rank's rows) or outside every
// head's vocabulary write zero rows, so a sum over the ranks assembles the
// full rows.  A row the host failed to read (flag set, or a NaN scale) is
// NaN in every channel, and the NaN survives that sum.
//
// One warp per row: the ring is staged in the warp's shared-memory slice,
// then each lane assembles the states of its channels from ceil(16/bits)
// fields, each read from a 32-bit window of two ring words.
// ============================================================================
namespace {

__device__ __forceinline__ float ple_code_value(uint32_t state) {
  const uint32_t p = state * 0x83DCD12Du;
  const uint32_t bytesum = __dp4a(p, 0x01010101u, 0u);
  // 0x6400 is fp16 1024 with a unit last place, so the sum lands exactly.
  const __half h = __ushort_as_half((unsigned short)(0x6400u + bytesum));
  const __half a = __ushort_as_half((unsigned short)0x1eee);
  const __half b = __ushort_as_half((unsigned short)0xc931);
  return __half2float(__hfma(h, a, b));
}

__device__ __forceinline__ int ple_head_of(int64_t id, const int64_t* __restrict__ off,
                                           const int64_t* __restrict__ vocab, int heads) {
  int lo = 0, hi = heads;  // first head starting after id
  while (lo < hi) {
    const int mid = (lo + hi) / 2;
    if (off[mid] <= id) lo = mid + 1;
    else hi = mid;
  }
  if (lo == 0) return -1;
  const int h = lo - 1;
  return (vocab[h] > 0 && id - off[h] < vocab[h]) ? h : -1;
}

__global__ void ple_decode_kernel(const uint16_t* __restrict__ rows, int64_t words, int ring_stride,
                                  const int64_t* __restrict__ ids, const __half* __restrict__ bias,
                                  const int64_t* __restrict__ head_off, const int64_t* __restrict__ head_vocab,
                                  int heads, int dim, int bits, int64_t owner_lo, int64_t owner_hi,
                                  const uint8_t* __restrict__ failed, __nv_bfloat16* __restrict__ out, int n) {
  extern __shared__ uint16_t ple_ring[];
  pdl_prologue();
  const int lane = threadIdx.x % 32, wpb = blockDim.x / 32;
  uint16_t* ring = ple_ring + (threadIdx.x / 32) * ring_stride;
  const int nw = (int)(words - 1);
  const uint32_t mask = (1u << bits) - 1u;
  for (int r = blockIdx.x * wpb + threadIdx.x / 32; r < n; r += gridDim.x * wpb) {
    const int64_t id = ids[r];
    __nv_bfloat16* o = out + (int64_t)r * dim;
    const int head = (id >= owner_lo && id < owner_hi) ? ple_head_of(id, head_off, head_vocab, heads) : -1;
    if (head < 0) {
      for (int c = lane; c < dim; c += 32) o[c] = __float2bfloat16_rn(0.f);
      continue;
    }
    const uint16_t* src = rows + (int64_t)r * words;
    float scale = __half2float(__ushort_as_half(src[0]));
    if (failed != nullptr && failed[r]) scale = __int_as_float(0x7fc00000);
    for (int i = lane; i < nw; i += 32) ring[i] = src[1 + i];
    __syncwarp();
    const __half* hb = bias + (int64_t)head * dim;
    for (int c = lane; c < dim; c += 32) {
      uint32_t state = 0;
      for (int g = 0; g * bits < 16; ++g) {
        const int ch = c >= g ? c - g : c - g + dim;
        const int p = ch * bits, w0 = p >> 4, w1 = w0 + 1 == nw ? 0 : w0 + 1;
        const uint32_t win = (uint32_t)ring[w0] | ((uint32_t)ring[w1] << 16);
        state |= ((win >> (p & 15)) & mask) << (g * bits);
      }
      const float v = ple_code_value(state & 0xffffu);
      o[c] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(v, scale), __half2float(hb[c])));
    }
    __syncwarp();
  }
}

}  // namespace

cudaError_t ple_decode_rows(const void* rows, int64_t words, const int64_t* ids, const void* bias,
                            const int64_t* head_off, const int64_t* head_vocab, int heads, int dim, int bits,
                            int64_t owner_lo, int64_t owner_hi, const uint8_t* failed, void* out, int n,
                            cudaStream_t stream) {
  if (bits < 1 || bits > 16 || dim <= 0 || heads <= 0 || ((int64_t)dim * bits) % 16 != 0 ||
      words != 1 + (int64_t)dim * bits / 16)
    return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int ring_stride = (int)(words / 2 * 2);  // words - 1 rounded up to even: 4-byte aligned slices
  const int64_t per_warp = (int64_t)ring_stride * 2;
  constexpr int64_t kSmemCap = 200 << 10;
  if (per_warp > kSmemCap) return cudaErrorInvalidValue;
  const int wpb = (int)std::min<int64_t>(8, kSmemCap / per_warp);
  const int smem = (int)(wpb * per_warp);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(ple_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  const int blocks = (int)std::min<int64_t>((n + wpb - 1) / wpb, 148 * 16);
  launch_pdl(ple_decode_kernel, dim3(blocks), dim3(32 * wpb), smem, stream, reinterpret_cast<const uint16_t*>(rows),
             words, ring_stride, ids, reinterpret_cast<const __half*>(bias), head_off, head_vocab, heads, dim, bits,
             owner_lo, owner_hi, failed, reinterpret_cast<__nv_bfloat16*>(out), n);
  return cudaGetLastError();
}

}  // namespace b200
