// Cross-GPU exchange and merge of split-KV decode partials over NVLink peer
// memory, in one kernel.
//
// Each rank owns an exchange buffer (the same size on every rank) that the
// other ranks map through CUDA IPC; its layout is in args.cuh (flags, the epoch,
// advanced on the device so a captured graph replays correctly, per-pair flags
// of the fused decode, and the fp32 (out, lse) slots of every source rank,
// double-buffered by epoch parity).
// One CTA per destination rank: CTA p writes the local partial into slot
// [parity][rank] of rank p's buffer (plain stores over NVLink, every
// destination in parallel), passes a barrier, and one thread fences at system
// scope and stores the epoch into rank p's flags[rank].  Every CTA then waits
// (bounded, relaxed polls and one fence) until all ranks' flags in its own
// buffer have reached the epoch and merges its share of the (request, head)
// rows exactly as the single-device merge does:
// o = sum_r 2^(lse_r - M) o_r / sum_r 2^(lse_r - M).
// Each CTA index has its own epoch word, advanced by that CTA at its end, so
// every CTA of a call reads the same epoch whatever order they start in.
//
// Slot reuse is safe with two parities: a rank overwrites parity p again only
// in call e + 2, after its call e + 1 has seen every peer's flag for e + 1,
// and each peer set that flag after its call e, which read parity p, had
// finished (calls are ordered on each rank's stream).
#include <type_traits>

#include "common.cuh"
#include "args.cuh"

namespace aicas {
namespace {

// 1024 threads: a CTA's push (one partial, 33 KB at config 5) and its share of
// the merge take one or two memory round trips per thread
constexpr int kExchangeThreads = 1024;

// four consecutive outputs in one store (8 bytes for 16-bit types)
template <typename T>
__device__ __forceinline__ void store4(T* p, float x, float y, float z, float w) {
  if constexpr (std::is_same<T, float>::value) {
    *reinterpret_cast<float4*>(p) = make_float4(x, y, z, w);
  } else {
    T v[4] = {Elem<T>::from_float(x), Elem<T>::from_float(y), Elem<T>::from_float(z), Elem<T>::from_float(w)};
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(v);
  }
}


template <typename T>
__global__ void __launch_bounds__(kExchangeThreads) exchange_merge_kernel(const ExchangeArgs a) {
  __shared__ int timed_out;
  // launched with programmatic dependent launch: the partials come from the
  // kernel before this one, and so (through it) does the previous call's epoch
  grid_dependency_wait();
  uint8_t* own = static_cast<uint8_t*>(a.peers[a.rank]);
  unsigned long long* flags = reinterpret_cast<unsigned long long*>(own);
  // this CTA's epoch word (one per CTA index: no CTA waits for another to
  // finish reading before the epoch can move)
  unsigned long long* epoch_word = reinterpret_cast<unsigned long long*>(own + 256) + blockIdx.x;
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(epoch_word) + 1;
  const int par = (int)(e & 1);
  const int nbh = a.batch * a.heads;
  const int n_o = nbh * a.hd;
  const int dst = blockIdx.x;  // destination rank of this CTA's push
  if (threadIdx.x == 0) timed_out = 0;

  // 1. publish the local partial into rank dst's buffer (own buffer for dst == rank)
  {
    float* slot = reinterpret_cast<float*>(static_cast<uint8_t*>(a.peers[dst]) + a.slot_off) +
                  ((size_t)par * a.world + a.rank) * a.slot_floats;
    const float4* src4 = reinterpret_cast<const float4*>(a.po);
    float4* dst4 = reinterpret_cast<float4*>(slot);
#pragma unroll 4
    for (int i = threadIdx.x; i < n_o / 4; i += blockDim.x) dst4[i] = __ldg(src4 + i);
    for (int i = threadIdx.x; i < nbh; i += blockDim.x) slot[n_o + i] = __ldg(a.plse + i);
  }
  // release: every thread's stores, the barrier, one system-scope fence, the flag
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    st_relaxed_sys(reinterpret_cast<unsigned long long*>(a.peers[dst]) + a.rank, e);
  }

  // 2. wait until every rank has published epoch e here (bounded), then acquire
  if (threadIdx.x < a.world) {
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t it = 1; ld_relaxed_sys(flags + threadIdx.x) < e; ++it) {
      if ((it & 63u) == 0u && global_timer_ns() - t0 > a.wait_budget_ns) {
        flag_device_error(a.err, AICAS_DEVERR_PEER_TIMEOUT);
        timed_out = 1;
        break;
      }
    }
    fence_acq_rel_sys();
  }
  __syncthreads();

  // 3. merge this CTA's share of the rows: one thread per (row, 4 columns)
  const float* slots = reinterpret_cast<const float*>(own + a.slot_off) + (size_t)par * a.world * a.slot_floats;
  const int q4 = a.hd / 4;
  const int rows_per = (nbh + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * rows_per, r1 = min(nbh, r0 + rows_per);
  for (int u = threadIdx.x; u < (r1 - r0) * q4; u += blockDim.x) {
    const int bh = r0 + u / q4, c4 = u % q4;
    const int b = bh / a.heads, h = bh % a.heads;
    // every rank's lse and columns read at once, from L2 (this SM's L1 may
    // hold the slot from two calls ago)
    float lse[kMaxExchangeRanks];
    float4 ov[kMaxExchangeRanks];
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxExchangeRanks; ++r) {
      const bool in = r < a.world && !timed_out;
      const float* sr = slots + (size_t)r * a.slot_floats;
      lse[r] = in ? __ldcg(sr + n_o + bh) : -INFINITY;
      ov[r] = in ? __ldcg(reinterpret_cast<const float4*>(sr + (size_t)bh * a.hd) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
      M = fmaxf(M, lse[r]);
    }
    float L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
#pragma unroll
      for (int r = 0; r < kMaxExchangeRanks; ++r) {
        const float w = exp2f(lse[r] - M);  // 0 for ranks past the world
        L += w;
        O.x = fmaf(w, ov[r].x, O.x);
        O.y = fmaf(w, ov[r].y, O.y);
        O.z = fmaf(w, ov[r].z, O.z);
        O.w = fmaf(w, ov[r].w, O.w);
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    T* orow = static_cast<T*>(a.out) + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + 4 * c4;
    store4<T>(orow, O.x * inv, O.y * inv, O.z * inv, O.w * inv);
    if (a.lse != nullptr && c4 == 0) a.lse[bh] = L > 0.f ? M + log2f(L) : -INFINITY;
  }

  // 4. this CTA's epoch word advances: the next call's CTA of the same index
  // reads it only after this grid has completed
  if (threadIdx.x == 0) *epoch_word = e;
}

}  // namespace

size_t exchange_slot_floats(int batch, int heads, int head_dim) {
  const size_t n = (size_t)batch * heads * (head_dim + 1);
  return (n + 3) & ~(size_t)3;  // keeps every slot 16-byte aligned
}

size_t exchange_buffer_bytes(int world, int batch, int heads, int head_dim) {
  return (size_t)exchange_slots_offset(batch, heads) +
         2 * (size_t)world * exchange_slot_floats(batch, heads, head_dim) * sizeof(float);
}

cudaError_t launch_exchange_merge(int dtype, const ExchangeArgs& a, cudaStream_t st) {
  const dim3 grid(a.world), block(kExchangeThreads);
  switch (dtype) {
    case AICAS_DTYPE_F32: return launch_pdl(exchange_merge_kernel<float>, grid, block, 0, st, a);
    case AICAS_DTYPE_F16: return launch_pdl(exchange_merge_kernel<__half>, grid, block, 0, st, a);
    case AICAS_DTYPE_BF16: return launch_pdl(exchange_merge_kernel<__nv_bfloat16>, grid, block, 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace aicas
