// NVFP4 quantiser for sm_100a: fp32 / fp16 / bf16 (L, rows, K) -> e2m1 codes (L, rows, K/2)
// and e4m3 block scales, written straight into the permuted ("blocked") layout the GEMM
// reads, optionally also in the plain (L, rows, K/16) layout.
//
// Semantics are the BASELINE input generation (restated in inputs.quantize_nvfp4):
//   scale_b = e4m3(amax(|x| over the 16-element block b) / 6)   (round to nearest even,
//                                                                out of range -> NaN)
//   v       = x / float(scale_b)   (correctly rounded; 0 when the scale is 0)
//   code    = nearest e2m1 of min(|v|, 6), ties to the even code; sign bit on non-zero codes
// The code comes from the hardware conversion cvt.rn.satfinite.e2m1x2.f32 (round to nearest,
// ties to even on the e2m1 grid, saturating at 6), with the -0 it gives for small negative
// values cleared to 0.
// Element 2i of a row goes to the low nibble of byte i.
//
// Layout of the permuted scales (kernels/gemm/reference.py:113-150): per 128-row block and
// 64-wide K block one 512-byte atom; row r, K-vector j at byte (r % 32) * 16 + (r / 32) * 4 + j.
// Rows past `rows` in the last block get scale 0, like the reference's padding.
//
// HBM-bound.  A CTA of 8 warps covers 128 rows x 4 atoms (256 elements of K); a warp
// takes 16 rows, and per row reads 256 contiguous elements with one 16-byte load per lane
// (two for fp32): lane l holds elements 8l .. 8l+7, half of 16-element block l/2, and
// the pair of lanes of a block reduces its amax with one shuffle.  Every load covers a
// whole 512-byte (1 KiB) stretch of one row, every code store 128 contiguous bytes; the
// CTA's scales are assembled in shared memory and leave as 2 KiB of whole atoms.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>

namespace nvfp4 {

enum QuantDtype : int { kQuantF32 = 0, kQuantF16 = 1, kQuantBF16 = 2 };

template <int DT>
__device__ __forceinline__ void load8(const void* src, float (&v)[8]) {
  if constexpr (DT == kQuantF32) {
    const float4* p = reinterpret_cast<const float4*>(src);
    const float4 f0 = __ldg(p), f1 = __ldg(p + 1);
    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f;
      if constexpr (DT == kQuantF16) f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// Two e2m1 codes from two floats with the hardware conversion: round to nearest, ties to
// the even code, saturating at +-6 (the reference's clamp), `lo` into the low nibble.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "cvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

constexpr int kQuantAtoms = 4;   // atoms (64 elements of K) per CTA
constexpr int kQuantRowsPerWarp = 16;
constexpr int kQuantBatch = 4;   // rows whose loads a warp keeps in flight together

// Codes of 8 elements (half a block) given the block's scale; returns 4 packed bytes.
// v = x / s is the correctly rounded division of the definition; negative values that
// round to zero keep code 0 (the conversion would give -0).
__device__ __forceinline__ uint32_t e2m1_pack8(const float (&v)[8], float s) {
  uint32_t w = 0;
  if (s > 0.f) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w |= cvt_e2m1x2(__fdiv_rn(v[2 * i], s), __fdiv_rn(v[2 * i + 1], s)) << (8 * i);
  }
  const uint32_t zero = ~(w | (w >> 1) | (w >> 2)) & 0x11111111u;  // magnitude-0 nibbles
  return w & ~(zero << 3);
}

// (4 CTAs of 8 warps per SM: other warps' loads cover a warp's compute phase)
template <int DT>
__global__ void __launch_bounds__(256, 4)
nvfp4_quantize_kernel(const void* __restrict__ x, int rows, int k, uint8_t* __restrict__ codes,
                      uint8_t* __restrict__ sf_perm, uint8_t* __restrict__ sf_plain) {
  __shared__ __align__(16) uint8_t atoms[kQuantAtoms * 512];
  constexpr int kElem = DT == kQuantF32 ? 4 : 2;
  const int rk = k / 64;
  const int rm = (rows + 127) / 128;
  const int kb0 = blockIdx.x * kQuantAtoms;  // first atom (64-wide K block) of this CTA
  const int n_atoms = min(kQuantAtoms, rk - kb0);
  const int rb = blockIdx.y;
  const int l = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kQuantAtoms * 512 / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(atoms)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  const int blk = lane >> 1;              // 16-element block within the 256 elements
  const int atom = blk >> 2, j = blk & 3;
  const bool lane_ok = atom < n_atoms;
  const int col = kb0 * 64 + lane * 8;    // first element of this lane
#pragma unroll 1
  for (int r0 = 0; r0 < kQuantRowsPerWarp; r0 += kQuantBatch) {
    float v[kQuantBatch][8];
#pragma unroll
    for (int b = 0; b < kQuantBatch; ++b) {
      const int r = warp * kQuantRowsPerWarp + r0 + b;
      const int row = rb * 128 + r;
      if (row < rows && lane_ok)
        load8<DT>(static_cast<const uint8_t*>(x) + (((long long)l * rows + row) * k + col) * kElem, v[b]);
      else
#pragma unroll
        for (int i = 0; i < 8; ++i) v[b][i] = 0.f;
    }
#pragma unroll
    for (int b = 0; b < kQuantBatch; ++b) {
      const int r = warp * kQuantRowsPerWarp + r0 + b;
      const int row = rb * 128 + r;
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[b][i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      if (row >= rows || !lane_ok) continue;
      const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(__fdiv_rn(amax, 6.0f), __NV_NOSAT, __NV_E4M3);
      const float s = float(*reinterpret_cast<const __nv_fp8_e4m3*>(&s8));
      const long long rowbase = (long long)l * rows + row;
      *reinterpret_cast<uint32_t*>(codes + (rowbase * k + col) / 2) = e2m1_pack8(v[b], s);
      if ((lane & 1) == 0) {
        atoms[atom * 512 + (r & 31) * 16 + (r >> 5) * 4 + j] = (uint8_t)s8;
        if (sf_plain) sf_plain[rowbase * (k / 16) + kb0 * 4 + blk] = (uint8_t)s8;
      }
    }
  }
  __syncthreads();
  // the CTA's atoms are consecutive in the permuted layout
  uint4* dst = reinterpret_cast<uint4*>(sf_perm + (((long long)l * rm + rb) * rk + kb0) * 512);
  for (int i = threadIdx.x; i < n_atoms * 512 / 16; i += blockDim.x)
    dst[i] = reinterpret_cast<const uint4*>(atoms)[i];
}

}  // namespace nvfp4
