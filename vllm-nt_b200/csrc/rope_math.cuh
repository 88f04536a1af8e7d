// NeoX rotation of one 16-byte vector pair, shared by the RoPE and the fused RoPE + KV-store
// kernels.
//
// Arithmetic mirrors vLLM's ApplyRotaryEmb.forward_static
// (vllm/model_executor/layers/rotary_embedding/common.py:144-183) op by op:
//   o1 = x1 * cos - x2 * sin,   o2 = x2 * cos + x1 * sin
// where each product and the final sum / difference is separately rounded (no FMA
// contraction) and, for 16-bit types, each torch op's result is rounded to the storage
// type.  16-bit elements are taken two at a time: the four products as paired 16-bit
// multiplies (see Mul2), the sum and difference in fp32, and one paired conversion per two
// results -- about half the instructions of an element-wise fp32 formulation, which matters
// because the rotation is issue-bound before it is HBM-bound.
#pragma once

#include "common.cuh"

namespace ntb200 {

// Two products of 16-bit values, each rounded once to the storage type.  The exact product
// of two bf16 (or two fp16) values fits in fp32's 24-bit significand, so rounding that fp32
// product to the storage type -- what torch's 16-bit multiply does -- is the single
// correctly rounded product the paired 16-bit multiply returns: one instruction for two
// products instead of two multiplies and a conversion.
template <typename T> struct Mul2;
template <> struct Mul2<__nv_bfloat16> {
  using W = __nv_bfloat162;
  static __device__ __forceinline__ W mul(W a, W b) { return __hmul2_rn(a, b); }
  static __device__ __forceinline__ float2 to_f2(W a) { return __bfloat1622float2(a); }
  static __device__ __forceinline__ W from_f2(float a, float b) { return __floats2bfloat162_rn(a, b); }
};
template <> struct Mul2<__half> {
  using W = __half2;
  static __device__ __forceinline__ W mul(W a, W b) { return __hmul2_rn(a, b); }
  static __device__ __forceinline__ float2 to_f2(W a) { return __half22float2(a); }
  static __device__ __forceinline__ W from_f2(float a, float b) { return __floats2half2_rn(a, b); }
};

template <typename T, int VEC>
__device__ __forceinline__ void rotate_vec(const Vec<T, VEC>& x1, const Vec<T, VEC>& x2, const Vec<T, VEC>& c,
                                           const Vec<T, VEC>& s, Vec<T, VEC>& o1, Vec<T, VEC>& o2) {
  if constexpr (sizeof(T) == 2 && VEC % 2 == 0) {
    using M = Mul2<T>;
    using W = typename M::W;
    const W* x1w = reinterpret_cast<const W*>(x1.v);
    const W* x2w = reinterpret_cast<const W*>(x2.v);
    const W* cw = reinterpret_cast<const W*>(c.v);
    const W* sw = reinterpret_cast<const W*>(s.v);
    W* o1w = reinterpret_cast<W*>(o1.v);
    W* o2w = reinterpret_cast<W*>(o2.v);
#pragma unroll
    for (int w = 0; w < VEC / 2; ++w) {
      const float2 a = M::to_f2(M::mul(x1w[w], cw[w]));  // x1 * cos
      const float2 b = M::to_f2(M::mul(x2w[w], sw[w]));  // x2 * sin
      const float2 e = M::to_f2(M::mul(x2w[w], cw[w]));  // x2 * cos
      const float2 f = M::to_f2(M::mul(x1w[w], sw[w]));  // x1 * sin
      o1w[w] = M::from_f2(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y));
      o2w[w] = M::from_f2(__fadd_rn(e.x, f.x), __fadd_rn(e.y, f.y));
    }
  } else {
    float r1[VEC], r2[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float xa = Elem<T>::to_f(x1.v[e]), xb = Elem<T>::to_f(x2.v[e]);
      const float ce = Elem<T>::to_f(c.v[e]), se = Elem<T>::to_f(s.v[e]);
      r1[e] = __fsub_rn(Elem<T>::round(__fmul_rn(xa, ce)), Elem<T>::round(__fmul_rn(xb, se)));
      r2[e] = __fadd_rn(Elem<T>::round(__fmul_rn(xb, ce)), Elem<T>::round(__fmul_rn(xa, se)));
    }
    o1 = pack_f<T, VEC>(r1);
    o2 = pack_f<T, VEC>(r2);
  }
}

}  // namespace ntb200
