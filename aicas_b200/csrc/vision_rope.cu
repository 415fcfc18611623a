// Vision-tower RoPE of q and k in one pass, straight from the packed QKV
// projection: HF apply_rotary_pos_emb_vision (transformers
// models/qwen3_vl/modeling_qwen3_vl.py:131-142), which the vision attention
// applies after splitting qkv (:205-209):
//     q_embed = (q.float() * cos) + (rotate_half(q.float()) * sin), then .to(dtype)
// with rotate_half(x) = cat(-x[D/2:], x[:D/2]) and cos/sin fp32 [T, D].  Every
// product and the sum are rounded as fp32 operations (no contraction into an
// FMA) and the result once to the dtype, so the output is bit-identical to the
// HF expression; HF runs it as about eight elementwise kernels per tensor over
// fp32 copies of q and k.
//
// A CTA takes whole tokens (grid-strided).  Each thread owns one 8-element chunk
// of the first half of one head row of q or k and the matching 8 of the second
// half, the same (q or k, head, chunk) for every token it visits, so the loop
// carries no index arithmetic beyond the token's row offsets: two 16-byte
// loads, two 16-byte stores, and the cos/sin values of both halves (fp32,
// shared by every head of the token, so they come from L1).  HBM-bound.
#include <algorithm>

#include "common.cuh"
#include "args.cuh"

namespace aicas {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) vision_rope_kernel(const VisionRopeArgs a) {
  const int chunks = a.hd >> 4;  // 8-element chunks per half row
  const int per_token = a.heads * 2 * chunks;
  const int half = a.hd / 2;
  grid_dependency_wait();
  for (int u = threadIdx.x; u < per_token; u += blockDim.x) {
    const int c = u % chunks;
    const int h = (u / chunks) % a.heads;
    const bool is_k = u >= chunks * a.heads;
    const T* src = static_cast<const T*>(is_k ? a.k_in : a.q_in) + (int64_t)h * (is_k ? a.ki_sh : a.qi_sh) + c * 8;
    T* dst = static_cast<T*>(is_k ? a.k_out : a.q_out) + (int64_t)h * (is_k ? a.ko_sh : a.qo_sh) + c * 8;
    const int64_t src_st = is_k ? a.ki_st : a.qi_st;
    const int64_t dst_st = is_k ? a.ko_st : a.qo_st;
    const float* cs0 = a.cos + c * 8;
    const float* sn0 = a.sin + c * 8;
    for (int t = blockIdx.x; t < a.tokens; t += gridDim.x) {
      const T* x = src + t * src_st;
      float x1[8], x2[8];
      Elem<T>::unpack(*reinterpret_cast<const uint4*>(x), x1);
      Elem<T>::unpack(*reinterpret_cast<const uint4*>(x + half), x2);
      const float* cs = cs0 + t * a.cs_st;
      const float* sn = sn0 + t * a.cs_st;
      float c1[8], c2[8], s1[8], s2[8];
#pragma unroll
      for (int e = 0; e < 8; e += 4) {
        *reinterpret_cast<float4*>(c1 + e) = __ldg(reinterpret_cast<const float4*>(cs + e));
        *reinterpret_cast<float4*>(c2 + e) = __ldg(reinterpret_cast<const float4*>(cs + half + e));
        *reinterpret_cast<float4*>(s1 + e) = __ldg(reinterpret_cast<const float4*>(sn + e));
        *reinterpret_cast<float4*>(s2 + e) = __ldg(reinterpret_cast<const float4*>(sn + half + e));
      }
      T y1[8], y2[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // (x * cos) + (rotate_half(x) * sin), each operation rounded in fp32
        y1[e] = Elem<T>::from_float(__fadd_rn(__fmul_rn(x1[e], c1[e]), __fmul_rn(-x2[e], s1[e])));
        y2[e] = Elem<T>::from_float(__fadd_rn(__fmul_rn(x2[e], c2[e]), __fmul_rn(x1[e], s2[e])));
      }
      T* y = dst + t * dst_st;
      *reinterpret_cast<uint4*>(y) = *reinterpret_cast<const uint4*>(y1);
      *reinterpret_cast<uint4*>(y + half) = *reinterpret_cast<const uint4*>(y2);
    }
  }
}

template <typename T>
cudaError_t launch_t(const VisionRopeArgs& a, int sms, cudaStream_t st) {
  const int per_token = a.heads * 2 * (a.hd >> 4);
  const int threads = per_token >= 256 ? 256 : (per_token + 31) / 32 * 32;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, vision_rope_kernel<T>, threads, 0);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  // one wave of resident CTAs, each striding over the tokens
  const long long blocks = std::min<long long>(a.tokens, (long long)sms * per_sm);
  return launch_pdl(vision_rope_kernel<T>, dim3((unsigned)blocks), dim3(threads), 0, st, a);
}

}  // namespace

cudaError_t launch_vision_rope(int dtype, const VisionRopeArgs& a, int sms, cudaStream_t st) {
  if (a.tokens == 0) return cudaSuccess;
  switch (dtype) {
    case AICAS_DTYPE_BF16: return launch_t<__nv_bfloat16>(a, sms, st);
    case AICAS_DTYPE_F16: return launch_t<__half>(a, sms, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace aicas
