// Fused (optional per-head RMSNorm) + rotate-half RoPE + KV-cache append.
//
// Semantics followed:
//   * RoPE: HF apply_rotary_pos_emb (transformers models/qwen3_vl/
//     modeling_qwen3_vl.py:410-432): x*cos + rotate_half(x)*sin with
//     rotate_half(x) = cat(-x[D/2:], x[:D/2]).  For 16-bit tensors every
//     elementwise product and the sum are rounded to the tensor dtype, exactly as
//     torch evaluates that expression on bf16/fp16 tensors, so the rotated q and
//     the cached k are bit-identical to the HF path for the same cos/sin.
//   * optional RMSNorm (Qwen3VLTextRMSNorm, modeling_qwen3_vl.py:390-407, and the
//     native fused kernel dujunbaoV1/native_cuda_ops/decode_q1_gqa_kernel.cu:376-480):
//     y = w * to_dtype(x * rsqrt(mean(x^2) + eps)).
//   * append: the in-place cache write of InplaceDecodeCacheLayer.update
//     (dujunbaoV1/evaluation_wrapper.py:84-100): token s of request b goes to
//     slot positions[b] + s; slots at or past the capacity are dropped, as the
//     reference truncates the payload at max_cache_len.
//
// One warp per (token, head row); q rows are written to q_out, k and v rows
// straight into their cache slot, so no intermediate tensor is materialised.
#include "common.cuh"
#include "args.cuh"

namespace aicas {

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return Elem<T>::to_float(Elem<T>::from_float(x));
}

// RoPE of one pair (x1 = x[j], x2 = x[j + D/2]) with the dtype's rounding.
template <typename T, bool kExactDtype>
__device__ __forceinline__ void rope_pair(float x1, float x2, float c1, float s1, float c2, float s2,
                                          float& y1, float& y2) {
  if (kExactDtype) {
    // y1 = x1*c1 + (-x2)*s1 ; y2 = x2*c2 + x1*s2, each op rounded to T
    const float a1 = round_to<T>(__fmul_rn(x1, c1));
    const float b1 = round_to<T>(__fmul_rn(-x2, s1));
    const float a2 = round_to<T>(__fmul_rn(x2, c2));
    const float b2 = round_to<T>(__fmul_rn(x1, s2));
    y1 = round_to<T>(__fadd_rn(a1, b1));
    y2 = round_to<T>(__fadd_rn(a2, b2));
  } else {
    y1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(-x2, s1));
    y2 = __fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2));
  }
}

template <typename T, typename CS>
__global__ void __launch_bounds__(128) rope_append_kernel(const RopeArgs a) {
  constexpr bool kExact = std::is_same<T, CS>::value;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x;  // b * seq + s
  const int b = row / a.seq, s = row % a.seq;
  const int slot_head = blockIdx.y * 4 + warp;
  const int nheads = a.hq + 2 * a.hkv;
  // launched with programmatic dependent launch: the attention that follows
  // may set up meanwhile; the inputs come from the kernel before this one
  grid_launch_dependents();
  grid_dependency_wait();
  if (a.kv_lens_out != nullptr && s == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    a.kv_lens_out[b] = min(max(a.positions[b], 0) + a.seq, a.cap);
  if (slot_head >= nheads) return;
  const int half = a.hd / 2;
  const CS* cp = static_cast<const CS*>(a.cos) + (int64_t)b * a.cs_sb + (int64_t)s * a.cs_ss;
  const CS* sp = static_cast<const CS*>(a.sin) + (int64_t)b * a.cs_sb + (int64_t)s * a.cs_ss;

  if (slot_head >= a.hq + a.hkv) {
    // value row: plain copy into the cache slot
    const int h = slot_head - a.hq - a.hkv;
    const int slot = a.positions[b] + s;
    if (slot < 0 || slot >= a.cap) return;
    const T* src = static_cast<const T*>(a.v_in) + (int64_t)b * a.v_sb + (int64_t)h * a.v_sh + (int64_t)s * a.v_ss;
    T* dst = static_cast<T*>(a.v_cache) + (int64_t)b * a.vc_sb + (int64_t)h * a.vc_sh + (int64_t)slot * a.hd;
    for (int j = lane; j < a.hd; j += 32) dst[j] = src[j];
    return;
  }

  const bool is_q = slot_head < a.hq;
  const int h = is_q ? slot_head : slot_head - a.hq;
  const T* src;
  T* dst;
  const T* w;
  if (is_q) {
    src = static_cast<const T*>(a.q_in) + (int64_t)b * a.qi_sb + (int64_t)h * a.qi_sh + (int64_t)s * a.qi_ss;
    dst = static_cast<T*>(a.q_out) + (int64_t)b * a.qo_sb + (int64_t)h * a.qo_sh + (int64_t)s * a.qo_ss;
    w = static_cast<const T*>(a.qw);
  } else {
    const int slot = a.positions[b] + s;
    if (slot < 0 || slot >= a.cap) return;
    src = static_cast<const T*>(a.k_in) + (int64_t)b * a.k_sb + (int64_t)h * a.k_sh + (int64_t)s * a.k_ss;
    dst = static_cast<T*>(a.k_cache) + (int64_t)b * a.kc_sb + (int64_t)h * a.kc_sh + (int64_t)slot * a.hd;
    w = static_cast<const T*>(a.kw);
  }

  // head_dim <= 128 -> at most 2 pairs per lane
  float x1[2], x2[2];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int j = lane + 32 * i;
    x1[i] = x2[i] = 0.f;
    if (j < half) {
      x1[i] = Elem<T>::to_float(src[j]);
      x2[i] = Elem<T>::to_float(src[j + half]);
      ss += x1[i] * x1[i] + x2[i] * x2[i];
    }
  }
  if (w != nullptr) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss / (float)a.hd + a.eps);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int j = lane + 32 * i;
      if (j < half) {
        const float w1 = Elem<T>::to_float(w[j]), w2 = Elem<T>::to_float(w[j + half]);
        x1[i] = round_to<T>(__fmul_rn(w1, round_to<T>(__fmul_rn(x1[i], inv))));
        x2[i] = round_to<T>(__fmul_rn(w2, round_to<T>(__fmul_rn(x2[i], inv))));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int j = lane + 32 * i;
    if (j < half) {
      const float c1 = Elem<CS>::to_float(cp[j]), c2 = Elem<CS>::to_float(cp[j + half]);
      const float s1 = Elem<CS>::to_float(sp[j]), s2 = Elem<CS>::to_float(sp[j + half]);
      float y1, y2;
      rope_pair<T, kExact>(x1[i], x2[i], c1, s1, c2, s2, y1, y2);
      dst[j] = Elem<T>::from_float(y1);
      dst[j + half] = Elem<T>::from_float(y2);
    }
  }
}

cudaError_t launch_rope_append(int dtype, int cs_dtype, const RopeArgs& a, cudaStream_t st) {
  const int nheads = a.hq + 2 * a.hkv;
  dim3 grid(a.batch * a.seq, (nheads + 3) / 4);
  const bool f32cs = cs_dtype == AICAS_DTYPE_F32;
  switch (dtype) {
    case AICAS_DTYPE_F32:
      return launch_pdl(rope_append_kernel<float, float>, grid, dim3(128), 0, st, a);
    case AICAS_DTYPE_F16:
      return f32cs ? launch_pdl(rope_append_kernel<__half, float>, grid, dim3(128), 0, st, a)
                   : launch_pdl(rope_append_kernel<__half, __half>, grid, dim3(128), 0, st, a);
    case AICAS_DTYPE_BF16:
      return f32cs ? launch_pdl(rope_append_kernel<__nv_bfloat16, float>, grid, dim3(128), 0, st, a)
                   : launch_pdl(rope_append_kernel<__nv_bfloat16, __nv_bfloat16>, grid, dim3(128), 0, st, a);
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ merge
// Combines P partial (o, lse) pairs: o = sum_p 2^(lse_p - M) o_p / sum_p 2^(lse_p - M).
template <typename T>
__global__ void __launch_bounds__(128) merge_partials_kernel(const MergeArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x * 4 + warp;
  if (bh >= a.batch * a.heads) return;
  const int b = bh / a.heads, h = bh % a.heads;
  const int64_t plane = (int64_t)a.batch * a.heads;
  float M = -INFINITY;
  for (int p = lane; p < a.np; p += 32) M = fmaxf(M, a.plse[p * plane + bh]);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float L = 0.f;
  if (M != -INFINITY)
    for (int p = 0; p < a.np; ++p) L += exp2f(a.plse[p * plane + bh] - M);
  for (int d = lane; d < a.hd; d += 32) {
    float O = 0.f;
    if (M != -INFINITY)
      for (int p = 0; p < a.np; ++p)
        O += exp2f(a.plse[p * plane + bh] - M) * a.po[(p * plane + bh) * a.hd + d];
    const float ov = L > 0.f ? O / L : 0.f;
    static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + d] = Elem<T>::from_float(ov);
  }
  if (a.lse != nullptr && lane == 0) a.lse[bh] = L > 0.f ? M + log2f(L) : -INFINITY;
}

cudaError_t launch_merge(int dtype, const MergeArgs& a, cudaStream_t st) {
  const int rows = a.batch * a.heads;
  dim3 grid((rows + 3) / 4);
  switch (dtype) {
    case AICAS_DTYPE_F32: merge_partials_kernel<float><<<grid, 128, 0, st>>>(a); break;
    case AICAS_DTYPE_F16: merge_partials_kernel<__half><<<grid, 128, 0, st>>>(a); break;
    case AICAS_DTYPE_BF16: merge_partials_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace aicas
