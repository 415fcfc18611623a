// Cross-GPU exchange and merge of split-KV decode partials over NVLink peer
// memory, in one kernel.
//
// Each rank owns an exchange buffer (the same size on every rank) that the
// other ranks map through CUDA IPC:
//   [0, 256)     uint64 flags[32]: flags[src] = last epoch rank src published here
//   [256, 264)   uint64 epoch: calls completed by the owner (advanced on the device,
//                so a captured graph replays correctly)
//   [512, ...)   fp32 slots[2][world][slot_floats]: the (out, lse) partial of each
//                source rank, double-buffered by epoch parity
// One CTA per call: it writes the local partial into slot [parity][rank] of
// every rank's buffer (plain stores over NVLink), fences at system scope and
// publishes the epoch with a release store into each peer's flags[rank];
// then it waits (bounded) until every rank's flag in its own buffer has
// reached the epoch, and merges the partials exactly as the single-device
// merge does: o = sum_r 2^(lse_r - M) o_r / sum_r 2^(lse_r - M).
//
// Slot reuse is safe with two parities: a rank overwrites parity p again only
// in call e + 2, after its call e + 1 has seen every peer's flag for e + 1,
// and each peer set that flag after its call e, which read parity p, had
// finished (calls are ordered on each rank's stream).
#include "common.cuh"
#include "args.cuh"

namespace aicas {
namespace {

constexpr int kExchangeThreads = 512;
constexpr size_t kSlotOffset = 512;

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kExchangeThreads) exchange_merge_kernel(const ExchangeArgs a) {
  __shared__ int timed_out;
  uint8_t* own = static_cast<uint8_t*>(a.peers[a.rank]);
  unsigned long long* flags = reinterpret_cast<unsigned long long*>(own);
  unsigned long long* epoch_word = reinterpret_cast<unsigned long long*>(own + 256);
  const unsigned long long e = *epoch_word + 1;
  const int par = (int)(e & 1);
  const int nbh = a.batch * a.heads;
  const int n_o = nbh * a.hd;
  if (threadIdx.x == 0) timed_out = 0;

  // 1. publish the local partial into every rank's buffer (own included)
  for (int p = 0; p < a.world; ++p) {
    float* dst = reinterpret_cast<float*>(static_cast<uint8_t*>(a.peers[p]) + kSlotOffset) +
                 ((size_t)par * a.world + a.rank) * a.slot_floats;
    const float4* src4 = reinterpret_cast<const float4*>(a.po);
    float4* dst4 = reinterpret_cast<float4*>(dst);
    for (int i = threadIdx.x; i < n_o / 4; i += blockDim.x) dst4[i] = src4[i];
    for (int i = threadIdx.x; i < nbh; i += blockDim.x) dst[n_o + i] = a.plse[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.world)
    st_release_sys(reinterpret_cast<unsigned long long*>(a.peers[threadIdx.x]) + a.rank, e);

  // 2. wait until every rank has published epoch e here (bounded)
  if (threadIdx.x < a.world) {
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t it = 1; ld_acquire_sys(flags + threadIdx.x) < e; ++it) {
      if ((it & 63u) == 0u && global_timer_ns() - t0 > kWaitBudgetNs) {
        flag_device_error(a.err, AICAS_DEVERR_PEER_TIMEOUT);
        timed_out = 1;
        break;
      }
    }
  }
  __syncthreads();

  // 3. merge: one warp per (request, head) row
  const float* slots = reinterpret_cast<const float*>(own + kSlotOffset) + (size_t)par * a.world * a.slot_floats;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int bh = warp; bh < nbh; bh += kExchangeThreads / 32) {
    const int b = bh / a.heads, h = bh % a.heads;
    float M = -INFINITY;
    if (!timed_out)
      for (int r = lane; r < a.world; r += 32) M = fmaxf(M, slots[(size_t)r * a.slot_floats + n_o + bh]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    if (M != -INFINITY)
      for (int r = 0; r < a.world; ++r) L += exp2f(slots[(size_t)r * a.slot_floats + n_o + bh] - M);
    for (int d = lane; d < a.hd; d += 32) {
      float O = 0.f;
      if (M != -INFINITY)
        for (int r = 0; r < a.world; ++r) {
          const float* s = slots + (size_t)r * a.slot_floats;
          O += exp2f(s[n_o + bh] - M) * s[(size_t)bh * a.hd + d];
        }
      const float ov = L > 0.f ? O / L : 0.f;
      static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + d] = Elem<T>::from_float(ov);
    }
    if (a.lse != nullptr && lane == 0) a.lse[bh] = L > 0.f ? M + log2f(L) : -INFINITY;
  }

  // 4. this call is complete on this rank
  __syncthreads();
  if (threadIdx.x == 0) *epoch_word = e;
}

}  // namespace

size_t exchange_slot_floats(int batch, int heads, int head_dim) {
  const size_t n = (size_t)batch * heads * (head_dim + 1);
  return (n + 3) & ~(size_t)3;  // keeps every slot 16-byte aligned
}

size_t exchange_buffer_bytes(int world, int batch, int heads, int head_dim) {
  return kSlotOffset + 2 * (size_t)world * exchange_slot_floats(batch, heads, head_dim) * sizeof(float);
}

cudaError_t launch_exchange_merge(int dtype, const ExchangeArgs& a, cudaStream_t st) {
  switch (dtype) {
    case AICAS_DTYPE_F32: exchange_merge_kernel<float><<<1, kExchangeThreads, 0, st>>>(a); break;
    case AICAS_DTYPE_F16: exchange_merge_kernel<__half><<<1, kExchangeThreads, 0, st>>>(a); break;
    case AICAS_DTYPE_BF16: exchange_merge_kernel<__nv_bfloat16><<<1, kExchangeThreads, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace aicas
