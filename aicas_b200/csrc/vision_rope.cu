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
// Each thread takes 8 elements of the first half of one (token, head) row of q
// or k and the matching 8 of the second half: two 16-byte loads, two 16-byte
// stores, and the cos/sin values of both halves (fp32, shared by every head of
// the token, so they come from L1/L2).  HBM-bound.
#include "common.cuh"
#include "args.cuh"

namespace aicas {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) vision_rope_kernel(const VisionRopeArgs a) {
  const int chunks = a.hd / 16;  // 8-element chunks per half row
  const long long total = (long long)a.tokens * a.heads * 2 * chunks;
  const int half = a.hd / 2;
  grid_dependency_wait();
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % chunks);
    long long rest = idx / chunks;
    const int h = (int)(rest % a.heads);
    rest /= a.heads;
    const int is_k = (int)(rest & 1);
    const long long t = rest >> 1;
    const T* src = static_cast<const T*>(is_k ? a.k_in : a.q_in) +
                   t * (is_k ? a.ki_st : a.qi_st) + (long long)h * (is_k ? a.ki_sh : a.qi_sh);
    T* dst = static_cast<T*>(is_k ? a.k_out : a.q_out) + t * (is_k ? a.ko_st : a.qo_st) +
             (long long)h * (is_k ? a.ko_sh : a.qo_sh);
    const int j = c * 8;
    float x1[8], x2[8];
    Elem<T>::unpack(*reinterpret_cast<const uint4*>(src + j), x1);
    Elem<T>::unpack(*reinterpret_cast<const uint4*>(src + j + half), x2);
    const float* cs = a.cos + t * a.cs_st;
    const float* sn = a.sin + t * a.cs_st;
    float c1[8], c2[8], s1[8], s2[8];
#pragma unroll
    for (int e = 0; e < 8; e += 4) {
      *reinterpret_cast<float4*>(c1 + e) = __ldg(reinterpret_cast<const float4*>(cs + j + e));
      *reinterpret_cast<float4*>(c2 + e) = __ldg(reinterpret_cast<const float4*>(cs + j + half + e));
      *reinterpret_cast<float4*>(s1 + e) = __ldg(reinterpret_cast<const float4*>(sn + j + e));
      *reinterpret_cast<float4*>(s2 + e) = __ldg(reinterpret_cast<const float4*>(sn + j + half + e));
    }
    T y1[8], y2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // (x * cos) + (rotate_half(x) * sin), each operation rounded in fp32
      y1[e] = Elem<T>::from_float(__fadd_rn(__fmul_rn(x1[e], c1[e]), __fmul_rn(-x2[e], s1[e])));
      y2[e] = Elem<T>::from_float(__fadd_rn(__fmul_rn(x2[e], c2[e]), __fmul_rn(x1[e], s2[e])));
    }
    *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(y1);
    *reinterpret_cast<uint4*>(dst + j + half) = *reinterpret_cast<const uint4*>(y2);
  }
}

}  // namespace

cudaError_t launch_vision_rope(int dtype, const VisionRopeArgs& a, int sms, cudaStream_t st) {
  const long long total = (long long)a.tokens * a.heads * 2 * (a.hd / 16);
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)sms * 8;  // grid-stride beyond eight blocks of 256 per SM
  if (blocks > cap) blocks = cap;
  switch (dtype) {
    case AICAS_DTYPE_BF16:
      return launch_pdl(vision_rope_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, st, a);
    case AICAS_DTYPE_F16:
      return launch_pdl(vision_rope_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, st, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace aicas
