// GQA decode attention (one query token per request) for sm_100a.
//
// Replaces the reference's Triton decode kernel
// (triton_qwen3vl/gqa_decode_attention.py:46-141, launcher :268-327) and the
// native fp16 kernel (dujunbaoV1/native_cuda_ops/decode_q1_gqa_kernel.cu:53-125).
// Same math: o = softmax(scale * q K^T) V with an fp32 online softmax in base 2,
// P rounded to the cache dtype before the PV product (gqa_decode_attention.py:128)
// and LSE = m + log2(l) in the base-2 scaled domain (:141).
//
// B200 design:
//   * one CTA per (request, KV head, split of the cache); the whole GQA group of
//     query heads is served from ONE copy of each K/V tile (the reference streams
//     the KV head once per query head);
//   * a producer warp streams 16 KB K and V tiles with cp.async.bulk (TMA into
//     this CTA's shared memory, L2 evict-first) into a 3-stage mbarrier ring;
//   * 4 consumer warps each own a quarter of every tile: 16-byte vector reads
//     from shared memory, a reduce-scatter of the q.k partial sums over the lanes
//     of a token, warp-shuffle maxima, per-warp online softmax;
//   * per-request lengths come from a device vector (no host synchronisation);
//   * the last CTA of a (request, KV head) merges the split partials (LSE merge)
//     and resets its counter, so one launch produces the final output.
#include "common.cuh"
#include "args.cuh"

namespace aicas {

template <typename T, int D, int G>
struct DecodeCfg {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kEPV = 16 / (int)sizeof(T);   // elements per 16-byte vector
  static constexpr int kLPT = D / kEPV;               // lanes per token
  static constexpr int kTPP = 32 / kLPT;              // tokens per warp pass
  static constexpr int kWarps = 4;                    // consumer warps
  static constexpr int kThreads = (kWarps + 1) * 32;  // + 1 producer warp
  static constexpr int kTileBytes = 16384;
  static constexpr int kTile = kTileBytes / kRowBytes;  // tokens per stage
  static constexpr int kTPW = kTile / kWarps;           // tokens per warp per tile
  static constexpr int kNP = kTPW / kTPP;               // passes per tile
  static constexpr int kNV = kNP * G;                   // partial scores per lane
  static constexpr int kLogLPT = kLPT == 1 ? 0 : kLPT == 2 ? 1 : kLPT == 4 ? 2 : kLPT == 8 ? 3 : kLPT == 16 ? 4 : 5;
  static constexpr int kLogNP = kNP == 8 ? 3 : -1;
  // halving steps of the reduce-scatter: stop once a lane holds one full pass (G values)
  static constexpr int kHalve = kLogLPT < kLogNP ? kLogLPT : kLogNP;
  static constexpr int kRV = kNV >> kHalve;            // values kept per lane (multiple of G)
  static constexpr int kDup = kLPT >> kHalve;          // lanes holding identical values
  static constexpr int kStages = 3;
  static constexpr int kRedFloats = kWarps * G * (D + 2);
  static constexpr int kPFloats = kTile * G;
  static constexpr int kSmemBytes = 2 * kStages * kTileBytes + 2 * kStages * 8 +
                                    (kRedFloats + kPFloats) * 4 + 16;
  static_assert(kEPV * kLPT == D, "head_dim must be a multiple of the vector width");
  static_assert(kLPT <= 32 && kTPP * kLPT == 32, "lanes per token must divide 32");
  static_assert(kNP == 8, "tile geometry");
  static_assert(kRV % G == 0, "each lane must keep whole passes");
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(DecodeCfg<T, D, G>::kThreads)
    decode_gqa_kernel(const DecodeArgs a) {
  using C = DecodeCfg<T, D, G>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sk = smem;
  uint8_t* sv = smem + C::kStages * C::kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * C::kStages * C::kTileBytes);
  float* red = reinterpret_cast<float*>(bars + 2 * C::kStages);  // [warp][G][D+2]
  float* ps = red + C::kRedFloats;                                // [tile token][G]
  __shared__ int s_abort;
  __shared__ int s_last;

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  int len = a.cap;
  if (a.kv_lens != nullptr) len = min(max(a.kv_lens[b], 0), a.cap);
  const int nsplit = max(1, (len + a.split_tokens - 1) / a.split_tokens);
  if (split >= nsplit) return;  // uniform for the CTA
  const int t0 = split * a.split_tokens;
  const int ntok = max(0, min(len, t0 + a.split_tokens) - t0);
  const int ntiles = (ntok + C::kTile - 1) / C::kTile;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + C::kStages);

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, C::kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const uint8_t* gk = static_cast<const uint8_t*>(a.k) +
                      ((int64_t)b * a.k_sb + (int64_t)kvh * a.k_sh + (int64_t)t0 * D) * sizeof(T);
  const uint8_t* gv = static_cast<const uint8_t*>(a.v) +
                      ((int64_t)b * a.v_sb + (int64_t)kvh * a.v_sh + (int64_t)t0 * D) * sizeof(T);

  float o[G][C::kEPV];
  float m[G], l[G];

  if (warp == C::kWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % C::kStages;
        const int u = t / C::kStages;
        if (t >= C::kStages && !mbar_wait(empty0 + 8 * s, (u - 1) & 1, &s_abort, a.err)) break;
        const uint32_t nb = (uint32_t)min(C::kTile, ntok - t * C::kTile) * C::kRowBytes;
        mbar_arrive_expect_tx(full0 + 8 * s, 2 * nb);
        bulk_g2s(smem_u32(sk + s * C::kTileBytes), gk + (int64_t)t * C::kTileBytes, nb, full0 + 8 * s, pol);
        bulk_g2s(smem_u32(sv + s * C::kTileBytes), gv + (int64_t)t * C::kTileBytes, nb, full0 + 8 * s, pol);
        ++issued;
      }
      if (s_abort) {
        // do not leave while our own copies may still land in shared memory
        for (int t = max(0, issued - C::kStages); t < issued; ++t)
          mbar_wait(full0 + 8 * (t % C::kStages), (t / C::kStages) & 1, nullptr, a.err);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int c = lane % C::kLPT;    // 16-byte column of the head_dim row
    const int sub = lane / C::kLPT;  // token slot within a pass
    const int gl = c;                // lane index inside its token group
    float qf[G][C::kEPV];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const T* qp = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)(kvh * G + h) * a.q_sh;
      const uint4 u = *reinterpret_cast<const uint4*>(qp + c * C::kEPV);
      Elem<T>::unpack(u, qf[h]);
#pragma unroll
      for (int e = 0; e < C::kEPV; ++e) qf[h][e] *= a.scale_log2;
      m[h] = -INFINITY;
      l[h] = 0.f;
#pragma unroll
      for (int e = 0; e < C::kEPV; ++e) o[h][e] = 0.f;
    }
    // index of the first value this lane keeps after the reduce-scatter
    int idx_base = 0;
#pragma unroll
    for (int k = 0; k < C::kHalve; ++k)
      if (gl & (C::kLPT >> (k + 1))) idx_base += C::kNV >> (k + 1);
    const bool canonical = (gl % C::kDup) == 0;
    float* pw = ps + warp * C::kTPW * G;  // this warp's probabilities [token][G]

    for (int t = 0; t < ntiles; ++t) {
      const int s = t % C::kStages;
      if (!mbar_wait(full0 + 8 * s, (t / C::kStages) & 1, &s_abort, a.err)) break;
      const uint8_t* tk = sk + s * C::kTileBytes;
      const uint8_t* tv = sv + s * C::kTileBytes;
      const int nvalid = min(C::kTile, ntok - t * C::kTile);
      const int wtok0 = warp * C::kTPW;  // first tile token of this warp

      // ---- scores: partial dot products over this lane's 16-byte column
      float sc[C::kNV];
#pragma unroll
      for (int p = 0; p < C::kNP; ++p) {
        const int tok = wtok0 + p * C::kTPP + sub;
        const uint4 u = *reinterpret_cast<const uint4*>(tk + tok * C::kRowBytes + c * 16);
        float kf[C::kEPV];
        Elem<T>::unpack(u, kf);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float acc = 0.f;
#pragma unroll
          for (int e = 0; e < C::kEPV; ++e) acc = fmaf(qf[h][e], kf[e], acc);
          sc[p * G + h] = acc;
        }
      }
      // ---- reduce-scatter across the kLPT lanes of a token, then butterfly
#pragma unroll
      for (int k = 0; k < C::kHalve; ++k) {
        const int off = C::kLPT >> (k + 1);
        const int half = C::kNV >> (k + 1);
        const bool upper = (gl & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = upper ? sc[i] : sc[i + half];
          const float keep = upper ? sc[i + half] : sc[i];
          sc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
#pragma unroll
      for (int k = C::kHalve; k < C::kLogLPT; ++k) {
        const int off = C::kLPT >> (k + 1);
#pragma unroll
        for (int i = 0; i < C::kRV; ++i) sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], off);
      }
      // lane now holds values idx_base .. idx_base + kRV - 1, i.e. passes
      // idx_base/G .. + kRV/G - 1 for every head; mask tokens past the split end
#pragma unroll
      for (int r = 0; r < C::kRV; ++r) {
        const int pass = (idx_base + r) / G;
        const int tok = wtok0 + pass * C::kTPP + sub;
        if (tok >= nvalid) sc[r] = -INFINITY;
      }
      // ---- online softmax, one state per warp and head
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float mt = -INFINITY;
#pragma unroll
        for (int r = h; r < C::kRV; r += G) mt = fmaxf(mt, sc[r]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
        const float m_new = fmaxf(m[h], mt);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        if (m_new != m[h]) {
          const float alpha = exp2f(m[h] - m_use);
          l[h] *= alpha;
#pragma unroll
          for (int e = 0; e < C::kEPV; ++e) o[h][e] *= alpha;
          m[h] = m_new;
        }
        float lsum = 0.f;
#pragma unroll
        for (int r = h; r < C::kRV; r += G) {
          const float p = exp2f(sc[r] - m_use);
          lsum += p;
          if (canonical) {
            const int pass = (idx_base + r) / G;
            pw[(pass * C::kTPP + sub) * G + h] = p;
          }
        }
        if (canonical) l[h] += lsum;
      }
      __syncwarp();
      // ---- o += P V over this lane's column (P rounded to the cache dtype)
#pragma unroll
      for (int p = 0; p < C::kNP; ++p) {
        const int wt = p * C::kTPP + sub;
        if (wtok0 + wt < nvalid) {
          const uint4 u = *reinterpret_cast<const uint4*>(tv + (wtok0 + wt) * C::kRowBytes + c * 16);
          float vf[C::kEPV];
          Elem<T>::unpack(u, vf);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float pr = Elem<T>::to_float(Elem<T>::from_float(pw[wt * G + h]));
#pragma unroll
            for (int e = 0; e < C::kEPV; ++e) o[h][e] = fmaf(pr, vf[e], o[h][e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
    }

    // ---- combine the token slots of the warp, then publish per-warp state
#pragma unroll
    for (int h = 0; h < G; ++h) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) l[h] += __shfl_xor_sync(0xffffffffu, l[h], off);
#pragma unroll
      for (int off = C::kLPT; off < 32; off <<= 1) {
#pragma unroll
        for (int e = 0; e < C::kEPV; ++e) o[h][e] += __shfl_xor_sync(0xffffffffu, o[h][e], off);
      }
      float* rw = red + (warp * G + h) * (D + 2);
      if (sub == 0) {
#pragma unroll
        for (int e = 0; e < C::kEPV; ++e) rw[c * C::kEPV + e] = o[h][e];
      }
      if (lane == 0) {
        rw[D] = m[h];
        rw[D + 1] = l[h];
      }
    }
  }
  __syncthreads();

  // ---- merge the consumer warps: result for (h, d) of this split
  const int bh = b * a.hkv + kvh;
  const bool single = (nsplit == 1);
  for (int idx = threadIdx.x; idx < G * D; idx += C::kThreads) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::kWarps; ++w) M = fmaxf(M, red[(w * G + h) * (D + 2) + D]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < C::kWarps; ++w) {
        const float* rw = red + (w * G + h) * (D + 2);
        const float sc = exp2f(rw[D] - M);
        L += rw[D + 1] * sc;
        O += rw[d] * sc;
      }
    }
    const float ov = (L > 0.f) ? O / L : 0.f;
    const float lse = (L > 0.f) ? M + log2f(L) : -INFINITY;
    const int qh = kvh * G + h;
    if (single) {
      if (a.out != nullptr)
        static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)qh * a.o_sh + d] = Elem<T>::from_float(ov);
      if (a.partial_o != nullptr) a.partial_o[((int64_t)b * a.hq + qh) * D + d] = ov;
      if (a.lse != nullptr && d == 0) a.lse[(int64_t)b * a.hq + qh] = lse;
    } else {
      a.ws_o[(((int64_t)bh * a.max_splits + split) * G + h) * D + d] = ov;
      if (d == 0) a.ws_lse[((int64_t)bh * a.max_splits + split) * G + h] = lse;
    }
  }
  if (single) return;

  // ---- split-KV: the last CTA of this (request, KV head) merges all splits
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(&a.ws_count[bh], 1u);
    s_last = (prev == (unsigned int)(nsplit - 1));
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  for (int idx = threadIdx.x; idx < G * D; idx += C::kThreads) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s)
      M = fmaxf(M, __ldcg(a.ws_lse + ((int64_t)bh * a.max_splits + s) * G + h));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < nsplit; ++s) {
        const int64_t base = ((int64_t)bh * a.max_splits + s) * G + h;
        const float w = exp2f(__ldcg(a.ws_lse + base) - M);
        L += w;
        O += w * __ldcg(a.ws_o + base * D + d);
      }
    }
    const float ov = (L > 0.f) ? O / L : 0.f;
    const float lse = (L > 0.f) ? M + log2f(L) : -INFINITY;
    const int qh = kvh * G + h;
    if (a.out != nullptr)
      static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)qh * a.o_sh + d] = Elem<T>::from_float(ov);
    if (a.partial_o != nullptr) a.partial_o[((int64_t)b * a.hq + qh) * D + d] = ov;
    if (a.lse != nullptr && d == 0) a.lse[(int64_t)b * a.hq + qh] = lse;
  }
  if (threadIdx.x == 0) a.ws_count[bh] = 0u;  // ready for the next call
}

// ------------------------------------------------------------------ host side

template <typename T, int D, int G>
static cudaError_t launch_decode_t(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  using C = DecodeCfg<T, D, G>;
  // the dynamic shared-memory opt-in is per function and per device
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(decode_gqa_kernel<T, D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  decode_gqa_kernel<T, D, G><<<grid, C::kThreads, C::kSmemBytes, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t dispatch_g(int g, const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  switch (g) {
    case 1: return launch_decode_t<T, D, 1>(a, grid, st);
    case 2: return launch_decode_t<T, D, 2>(a, grid, st);
    case 4: return launch_decode_t<T, D, 4>(a, grid, st);
    case 8: return launch_decode_t<T, D, 8>(a, grid, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t dispatch_d(int d, int g, const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  switch (d) {
    case 16: return dispatch_g<T, 16>(g, a, grid, st);
    case 32: return dispatch_g<T, 32>(g, a, grid, st);
    case 64: return dispatch_g<T, 64>(g, a, grid, st);
    case 128: return dispatch_g<T, 128>(g, a, grid, st);
  }
  return cudaErrorInvalidValue;
}

// tokens per stage: 16 KB of rows
int decode_tile_for(int dtype, int head_dim) {
  const int elem = dtype == AICAS_DTYPE_F32 ? 4 : 2;
  return 16384 / (head_dim * elem);
}

cudaError_t launch_decode(int dtype, int head_dim, int group, const DecodeArgs& a, cudaStream_t st) {
  dim3 grid(a.max_splits, a.hkv, a.batch);
  switch (dtype) {
    case AICAS_DTYPE_F32: return dispatch_d<float>(head_dim, group, a, grid, st);
    case AICAS_DTYPE_F16: return dispatch_d<__half>(head_dim, group, a, grid, st);
    case AICAS_DTYPE_BF16: return dispatch_d<__nv_bfloat16>(head_dim, group, a, grid, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace aicas
