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
