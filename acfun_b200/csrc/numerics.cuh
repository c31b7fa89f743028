// numerics.cuh — operand splitting for fp32 math on tensor cores.
//   3xTF32: x -> (tf32(x), tf32(x - tf32(x))), both stored as fp32 bit patterns
//   3xBF16: x -> (bf16(x), bf16(x - bf16(x))), stored as bf16
// Rounding is to nearest even; Inf / NaN pass through the high part.
#pragma once
#include <stdint.h>

namespace acf {

static __device__ __forceinline__ float nx_tf32_rne(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  u += 0xfffu + ((u >> 13) & 1u);
  return __uint_as_float(u & 0xffffe000u);
}

static __device__ __forceinline__ uint16_t nx_bf16_rne(float f) {
  const uint32_t x = __float_as_uint(f);
  if ((x & 0x7f800000u) == 0x7f800000u) return (uint16_t)((x >> 16) | ((x & 0xffffu) ? 0x40u : 0u));
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

static __device__ __forceinline__ float nx_bf16_val(uint16_t h) {
  return __uint_as_float((uint32_t)h << 16);
}

// Block-wide copy into shared memory, dst[i] = f(i) for i < n, each thread issuing its U
// loads before its U stores: one memory round trip per U*blockDim elements rather than one
// per blockDim.
template <int U, typename F>
static __device__ __forceinline__ void stage_block(float* dst, int n, F f) {
  for (int b0 = threadIdx.x; b0 < n; b0 += U * blockDim.x) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = b0 + u * blockDim.x;
      v[u] = i < n ? f(i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = b0 + u * blockDim.x;
      if (i < n) dst[i] = v[u];
    }
  }
}

// Running maximum of |v| as the int8 router's absmax accumulates it (k_absmax_img: a NaN never
// replaces the running value).
static __device__ __forceinline__ void amax_acc(float& am, float v) {
  const float a = fabsf(v);
  am = (am < a) ? a : am;
}

// 3xBF16 split of a pair on the hardware converter (cvt.rn.bf16x2.f32 rounds to nearest
// even, the same bits as nx_bf16_rne for every non-NaN input): hi = bf16(a) | bf16(b) << 16,
// lo = the bf16 of the exact remainders a - hi, b - hi in the same packing.
static __device__ __forceinline__ void nx_split_bf16x2(float a, float b, uint32_t& hi,
                                                       uint32_t& lo) {
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(b), "f"(a));
  const float ra = a - __uint_as_float(hi << 16), rb = b - __uint_as_float(hi & 0xffff0000u);
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(rb), "f"(ra));
}

// Store the split of 4 consecutive values at element index 4*i of the hi plane and the same
// index of the lo plane (op_stride elements further).
template <bool BF>
static __device__ __forceinline__ void nx_store_split4(void* dst, size_t i4, size_t op_stride,
                                                       const float (&v)[4]) {
  if constexpr (BF) {
    uint32_t h0, l0, h1, l1;
    nx_split_bf16x2(v[0], v[1], h0, l0);
    nx_split_bf16x2(v[2], v[3], h1, l1);
    uint16_t* d = reinterpret_cast<uint16_t*>(dst) + 4 * i4;
    *reinterpret_cast<uint2*>(d) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(d + op_stride) = make_uint2(l0, l1);
  } else {
    float h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h[k] = nx_tf32_rne(v[k]);
      l[k] = nx_tf32_rne(v[k] - h[k]);
    }
    float* d = reinterpret_cast<float*>(dst) + 4 * i4;
    *reinterpret_cast<float4*>(d) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(d + op_stride) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// Scalar store of one split value at element index i.
template <bool BF>
static __device__ __forceinline__ void nx_store_split1(void* dst, size_t i, size_t op_stride, float x) {
  if constexpr (BF) {
    const uint16_t h = nx_bf16_rne(x);
    uint16_t* d = reinterpret_cast<uint16_t*>(dst) + i;
    d[0] = h;
    d[op_stride] = nx_bf16_rne(x - nx_bf16_val(h));
  } else {
    const float h = nx_tf32_rne(x);
    float* d = reinterpret_cast<float*>(dst) + i;
    d[0] = h;
    d[op_stride] = nx_tf32_rne(x - h);
  }
}

// Two independent IEEE fma.rn in one instruction (sm_100 packed f32x2): lane k of the result
// is fmaf(a_k, b_k, c_k), bit-identical to __fmaf_rn on each lane.
static __device__ __forceinline__ float2 nx_ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d = __builtin_bit_cast(unsigned long long, c);
  asm("fma.rn.f32x2 %0, %1, %2, %0;"
      : "+l"(d)
      : "l"(__builtin_bit_cast(unsigned long long, a)), "l"(__builtin_bit_cast(unsigned long long, b)));
  return __builtin_bit_cast(float2, d);
}

}  // namespace acf
