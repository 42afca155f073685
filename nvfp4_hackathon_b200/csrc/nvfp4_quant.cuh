// NVFP4 quantiser for sm_100a: fp32 / fp16 / bf16 (L, rows, K) -> e2m1 codes (L, rows, K/2)
// and e4m3 block scales, written straight into the permuted ("blocked") layout the GEMM
// reads, optionally also in the plain (L, rows, K/16) layout.
//
// Semantics are the BASELINE input generation (restated in inputs.quantize_nvfp4):
//   scale_b = e4m3(amax(|x| over the 16-element block b) / 6)   (round to nearest even,
//                                                                out of range -> NaN)
//   v       = x / float(scale_b)   (correctly rounded; 0 when the scale is 0)
//   code    = nearest e2m1 of min(|v|, 6), ties to the even code; sign bit on non-zero codes
// v is formed exactly with one multiply and two fmas (Markstein's correction step, see
// quotient_rn); the code comes from the hardware conversion cvt.rn.satfinite.e2m1x2.f32
// (round to nearest, ties to even on the e2m1 grid, saturating at 6), with the -0 it gives
// for small negative values cleared to 0.
// Element 2i of a row goes to the low nibble of byte i.
//
// Layout of the permuted scales (kernels/gemm/reference.py:113-150): per 128-row block and
// 64-wide K block one 512-byte atom; row r, K-vector j at byte (r % 32) * 16 + (r / 32) * 4 + j.
// Rows past `rows` in the last block get scale 0, like the reference's padding.
//
// HBM-bound.  A CTA of 8 warps covers 128 rows x (32 lanes x 32 bytes) of input; a warp
// takes 16 rows, and per row each lane reads 32 contiguous bytes: 16 elements (one block)
// of fp16/bf16, or 8 fp32 elements (half a block; the pair of lanes reduces the block's amax
// with one shuffle).  Every load instruction covers 512 contiguous bytes of one row, the
// code stores are contiguous too, and the CTA's scales are assembled in shared memory and
// leave as whole atoms (4 or 8 of them).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>

namespace nvfp4 {

enum QuantDtype : int { kQuantF32 = 0, kQuantF16 = 1, kQuantBF16 = 2 };

// 32 bytes of input (two 16-byte vectors already in registers) -> 8 or 16 floats: fp32
// uses both vectors for 8 values; 16-bit types use one vector per 8 values.
template <int DT>
__device__ __forceinline__ void load8(const uint4* src, float (&v)[8]) {
  if constexpr (DT == kQuantF32) {
    const uint4 a = src[0], b = src[1];
    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y); v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
    v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y); v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
  } else {
    const uint4 u = src[0];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (DT == kQuantF16) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      } else {  // bf16 is the upper half of an fp32: widening is exact
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      }
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

constexpr int kQuantRowsPerWarp = 16;
constexpr int kQuantBatch = 4;   // rows whose loads a warp keeps in flight together
// Elements per lane: 32 bytes of input each, so fp32 lanes hold half a 16-element block
// (pairs of lanes reduce the block's amax) and 16-bit lanes a whole block.
template <int DT> __host__ __device__ constexpr int quant_epl() { return DT == kQuantF32 ? 8 : 16; }
template <int DT> __host__ __device__ constexpr int quant_atoms() { return quant_epl<DT>() / 2; }  // atoms per CTA

// Codes of 8 elements (half a block) given the block's scale and its correctly rounded
// reciprocal inv = RN(1/s); returns 4 packed bytes.  The definition rounds the correctly
// rounded quotient v = RN(x / s).  It is formed with Markstein's correction step
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990; J.-M. Muller et al., Handbook of
// Floating-Point Arithmetic, the theorem on division with a correctly rounded reciprocal):
//   q = RN(x * inv)            within one ulp of x / s
//   r = RN(x - q * s)          exact (one fma), since q is that close
//   v = RN(q + r * inv)        = RN(x / s)
// The theorem needs a normal quotient; any |x / s| below the first e2m1 threshold (0.25)
// gives code 0 whether or not it is exact, and the block's amax bounds |x / s| near 6,
// so every quotient that decides a code is in range.  No branch, one conversion per pair.
// Negative values that round to zero keep code 0 (the conversion would give -0).
__device__ __forceinline__ float quotient_rn(float x, float s, float inv) {
  const float q = __fmul_rn(x, inv);
  const float r = __fmaf_rn(-q, s, x);
  return __fmaf_rn(r, inv, q);
}

// The same three steps on two values at once with the packed fp32 instructions of sm_100
// (mul/fma .rn.f32x2: each half rounds exactly like the scalar instruction, so the results
// are bit for bit those of quotient_rn); ns = -s.
__device__ __forceinline__ void quotient_rn2(float x0, float x1, float ns, float inv, float& v0,
                                             float& v1) {
  uint64_t X, NS, INV, Q, R, V;
  asm("mov.b64 %0, {%1, %2};" : "=l"(X) : "f"(x0), "f"(x1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(NS) : "f"(ns));
  asm("mov.b64 %0, {%1, %1};" : "=l"(INV) : "f"(inv));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(Q) : "l"(X), "l"(INV));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(R) : "l"(Q), "l"(NS), "l"(X));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(V) : "l"(R), "l"(INV), "l"(Q));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v0), "=f"(v1) : "l"(V));
}

__device__ __forceinline__ uint32_t e2m1_pack8(const float (&v)[8], float s, float inv) {
  uint32_t w = 0;
  if (s > 0.f) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float q0, q1;
      quotient_rn2(v[2 * i], v[2 * i + 1], -s, inv, q0, q1);
      w |= cvt_e2m1x2(q0, q1) << (8 * i);
    }
  }
  const uint32_t zero = ~(w | (w >> 1) | (w >> 2)) & 0x11111111u;  // magnitude-0 nibbles
  return w & ~(zero << 3);
}

// (4 CTAs of 8 warps per SM: other warps' loads cover a warp's compute phase)
template <int DT>
__global__ void __launch_bounds__(256, 4)
nvfp4_quantize_kernel(const void* __restrict__ x, int rows, int k, uint8_t* __restrict__ codes,
                      uint8_t* __restrict__ sf_perm, uint8_t* __restrict__ sf_plain) {
  constexpr int EPL = quant_epl<DT>();
  constexpr int ATOMS = quant_atoms<DT>();
  __shared__ __align__(16) uint8_t atoms[ATOMS * 512];
  constexpr int kElem = DT == kQuantF32 ? 4 : 2;
  const int rk = k / 64;
  const int rm = (rows + 127) / 128;
  const int kb0 = blockIdx.x * ATOMS;  // first atom (64-wide K block) of this CTA
  const int n_atoms = min(ATOMS, rk - kb0);
  const int rb = blockIdx.y;
  const int l = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < ATOMS * 512 / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(atoms)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  const int blk = lane * EPL / 16;        // 16-element block within the CTA's columns
  const int atom = blk >> 2, j = blk & 3;
  const bool lane_ok = atom < n_atoms;
  const int col = kb0 * 64 + lane * EPL;  // first element of this lane
  const bool writer = EPL == 16 || (lane & 1) == 0;
#pragma unroll 1
  for (int r0 = 0; r0 < kQuantRowsPerWarp; r0 += kQuantBatch) {
    // raw loads in flight (32 bytes per lane and row, whatever the type), converted later
    uint4 raw[kQuantBatch][2];
#pragma unroll
    for (int b = 0; b < kQuantBatch; ++b) {
      const int r = warp * kQuantRowsPerWarp + r0 + b;
      const int row = rb * 128 + r;
      const uint4* src = reinterpret_cast<const uint4*>(
          static_cast<const uint8_t*>(x) + (((long long)l * rows + row) * k + col) * kElem);
      if (row < rows && lane_ok) {
        raw[b][0] = __ldg(src);
        raw[b][1] = __ldg(src + 1);
      } else {
        raw[b][0] = raw[b][1] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int b = 0; b < kQuantBatch; ++b) {
      const int r = warp * kQuantRowsPerWarp + r0 + b;
      const int row = rb * 128 + r;
      float v[EPL];
      load8<DT>(&raw[b][0], *reinterpret_cast<float(*)[8]>(&v[0]));
      if constexpr (EPL == 16) load8<DT>(&raw[b][1], *reinterpret_cast<float(*)[8]>(&v[8]));
      float amax = 0.f;
      if constexpr (DT == kQuantF32) {
#pragma unroll
        for (int i = 0; i < EPL; ++i) amax = fmaxf(amax, fabsf(v[i]));
      } else {
        // |x| of two 16-bit values at once (clear both sign bits), then a max tree of packed
        // maxima: exact, and like fmaxf a NaN operand yields the other one
        const uint32_t w[8] = {raw[b][0].x, raw[b][0].y, raw[b][0].z, raw[b][0].w,
                               raw[b][1].x, raw[b][1].y, raw[b][1].z, raw[b][1].w};
        uint32_t m = w[0] & 0x7fff7fffu;
#pragma unroll
        for (int i = 1; i < 8; ++i) {
          const uint32_t a = w[i] & 0x7fff7fffu;
          if constexpr (DT == kQuantBF16) asm("max.bf16x2 %0, %0, %1;" : "+r"(m) : "r"(a));
          else asm("max.f16x2 %0, %0, %1;" : "+r"(m) : "r"(a));
        }
        float lo, hi;
        if constexpr (DT == kQuantBF16) {
          lo = __uint_as_float(m << 16);
          hi = __uint_as_float(m & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&m));
          lo = f.x;
          hi = f.y;
        }
        amax = fmaxf(lo, hi);
      }
      if constexpr (EPL == 8) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      if (row >= rows || !lane_ok) continue;
      // amax / 6 correctly rounded (1.0f / 6.0f folds to RN(1/6) at compile time; a
      // quotient too small for the correction step's theorem is below e4m3's range and
      // becomes scale 0 either way)
      const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(quotient_rn(amax, 6.0f, 1.0f / 6.0f), __NV_NOSAT, __NV_E4M3);
      const float s = float(*reinterpret_cast<const __nv_fp8_e4m3*>(&s8));
      const float inv = s > 0.f ? __frcp_rn(s) : 0.f;  // correctly rounded 1 / s
      const long long rowbase = (long long)l * rows + row;
      uint8_t* cdst = codes + (rowbase * k + col) / 2;
      if constexpr (EPL == 16) {
        float lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) { lo[i] = v[i]; hi[i] = v[8 + i]; }
        *reinterpret_cast<uint2*>(cdst) = make_uint2(e2m1_pack8(lo, s, inv), e2m1_pack8(hi, s, inv));
      } else {
        float h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = v[i];
        *reinterpret_cast<uint32_t*>(cdst) = e2m1_pack8(h, s, inv);
      }
      if (writer) {
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
