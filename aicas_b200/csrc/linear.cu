// Decode-side weight-streaming products on the sm_100a tensor cores:
//   Y[R, N] = epilogue(X'[R, K] W[N, K]^T),  R <= 32 rows (one decode step's batch)
// with X' = X or HF's RMSNorm of X, and the epilogue a plain store, a residual
// add or SiLU(gate) * up.
//
// Replaces the matrix-vector kernels of the reference's native decode path
// (dujunbaoV1/native_cuda_ops/decode_q1_gqa_kernel.cu): rmsnorm_kernel
// :127-157 (here the prologue), gate_up_silu_matvec_kernel :174-220,
// dual_linear_matvec_kernel :222-269, qkv_linear_matvec_kernel :271-331 and
// the product half of lm_head_argmax_stage1_kernel :482-532.  Those run one
// warp per output feature on the CUDA cores; this kernel puts the weights on
// the MMA's M side instead: a 128-feature x 64-K weight tile is the A operand
// (TMA, 128-byte swizzle), the batch rows padded to RP (16 or 32) are the
// B operand, and the fp32 accumulator [128 features x RP rows] sits in TMEM.
// The tensor cores are idle most of the time; the kernel is bound by the
// weight stream from HBM.
//
// Work split ("stream-K"): the (tile, 64-K block) units of all output tiles
// are cut into `grid` equal contiguous ranges, one per CTA (grid <= SMs, one
// wave).  A CTA streams its units through a ring of shared-memory stages; a
// tile that lies wholly inside one CTA's range is finished by that CTA, a tile
// shared by several CTAs is finished by the last of them to arrive (a counter
// per tile), which adds the fp32 partials in CTA order, so the result does not
// depend on timing.  The counters are left at zero for the next call.
//
// Warp roles (192 threads):
//   warps 0-3  prologue (RMSNorm statistics, X' into shared memory in the MMA
//              layout) and epilogue (one TMEM lane = one output feature)
//   warp 4     TMA producer of the weight tiles
//   warp 5     TMEM allocation and the MMA-issuing thread
// Launched with programmatic dependent launch: the weight stream starts before
// the previous kernel on the stream has finished; only the prologue and the
// epilogue (activations, outputs, workspace) wait for it.  Dependents are
// released once a CTA has issued its last product.
#include <cuda.h>

#include <cstdio>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "linear.cuh"
#include "tcgen05.cuh"
#include "tma_host.cuh"

namespace aicas {
namespace {

constexpr int kTileN = 128;                       // output features per tile (MMA M)
constexpr int kKBlock = 64;                       // K elements per stage: one 128-byte swizzle row
constexpr int kTileBytes = kTileN * kKBlock * 2;  // 16 KB
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kSmemBudget = 232448 - 1024;  // opt-in shared memory per CTA on sm_100, less the static part
// Dynamic shared memory that lets two CTAs share an SM (228 KB per SM, 1 KB
// reserved per CTA, the static part): the next product's CTAs, launched early
// by programmatic dependent launch, then stream their weights while this
// kernel finishes.
constexpr int kSmemTwoPerSm = 112 << 10;
constexpr int kMaxStages = 8;
// The tile counters sit in a fixed region at the start of every workspace, so
// calls of different shapes can share one workspace: a call's partials never
// land on another call's counters.
constexpr size_t kCounterRegion = 64 << 10;
// the last slot counts the CTAs that finished (the sumsq_out epilogue)
constexpr int kDoneSlot = (int)(kCounterRegion / 4) - 1;
constexpr int kMaxTiles = kDoneSlot;
// Weights brought into L2 ahead of the ring, per call (the ring's loads then
// hit L2 while HBM streams the next product's weights): at most this many bytes.
constexpr long long kL2PrefetchBytes = 48ll << 20;

struct LinSeg {
  CUtensorMap tm;  // 2-D [rows, K], box {64, 128}, 128-byte swizzle
  void* out;
  int64_t out_stride;
  int rows;
  int tile0;  // first tile index of the segment
};

struct LinearArgs {
  LinSeg seg[AICAS_LINEAR_MAX_SEGMENTS];
  CUtensorMap tm_x;  // x' [R, K], box {64, RP} (rows past R read as zeros); used when x_tma
  int x_tma;         // 1: x is copied into the slots by TMA (then normalised in place when norm_w is set)
  float* sumsq_out;  // per-row sums of squares of the output of segment 0 (last CTA)
  const float* x_sumsq;  // per-row sums of squares of x (with norm_w: no statistics pass)
  const void* x;
  int64_t x_stride;
  const void* norm_w;
  const void* res;
  int64_t res_stride;
  float eps;
  int R, K, KB, nseg, mode, tiles, grid, stages, n_slots;
  int pf_units;  // units per CTA prefetched into L2 at entry
  int cs;        // 0: stream-K ranges; >= 1: tile blockIdx / cs, K split cs ways (a CTA cluster)
  int recv_bytes;  // cluster split: shared memory receiving the other CTAs' partials
  long long units;
  float* ss_part;  // sumsq_out: [shares][RP] per tile (stream-K) or per CTA (cluster split)
  uint32_t* counters;  // [tiles] at the start of the workspace
  float* partials;     // [2 * grid][P][RP][128]
  unsigned int* err;
};

__device__ __forceinline__ long long unit_begin(const LinearArgs& a, int c) {
  return (long long)c * a.units / a.grid;
}
// the CTA whose range holds unit u: the largest c with unit_begin(c) <= u
__device__ __forceinline__ int cta_of_unit(const LinearArgs& a, long long u) {
  return (int)(((u + 1) * a.grid - 1) / a.units);
}
// a CTA's partial of a shared tile: slot 0 for the first tile of its range, 1 for the last
__device__ __forceinline__ int partial_slot(const LinearArgs& a, int c, int t) {
  return 2 * c + ((long long)t == unit_begin(a, c) / a.KB ? 0 : 1);
}
__device__ __forceinline__ int seg_of_tile(const LinearArgs& a, int t) {
  int s = 0;
#pragma unroll
  for (int j = 1; j < AICAS_LINEAR_MAX_SEGMENTS; ++j)
    if (j < a.nseg && t >= a.seg[j].tile0) s = j;
  return s;
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// true on every epilogue thread iff pred holds on all of them
__device__ __forceinline__ bool epi_all(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u)
      : "memory");
  return r != 0;
}

// Cluster split: address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// Every thread of every CTA in the cluster calls this once, warps converged.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ unsigned int atom_add_acq_rel(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return Elem<T>::to_float(Elem<T>::from_float(v));
}

// HF Qwen3VLTextRMSNorm statistics of R rows of K elements (mean of squares
// in fp32) by the 128 epilogue threads: thread tid takes 8-element chunks tid,
// tid + 128, ... of every row, eight rows' loads in flight at once, then a
// block reduction per row.  rstd[r] = rsqrt(mean + eps).
template <typename T, bool kL2Only>
__device__ __forceinline__ void block_rstd(const T* x, int64_t stride, int R, int K, float eps, float* rstd,
                                           float (*red)[8]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int r0 = 0; r0 < R; r0 += 8) {
    float ss[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) ss[q] = 0.f;
#pragma unroll 2
    for (int k = tid * 8; k < K; k += kEpiThreads * 8) {
      uint4 v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (r0 + q < R) {
          const uint4* src = reinterpret_cast<const uint4*>(x + (r0 + q) * stride + k);
          v[q] = kL2Only ? __ldcg(src) : *src;
        }
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (r0 + q < R) {
          float f[8];
          Elem<T>::unpack(v[q], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss[q] = fmaf(f[e], f[e], ss[q]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss[q] += __shfl_xor_sync(0xffffffffu, ss[q], o);
      if (lane == 0) red[warp][q] = ss[q];
    }
    epi_sync();
    if (tid < 8 && r0 + tid < R)
      rstd[r0 + tid] = rsqrtf((red[0][tid] + red[1][tid] + red[2][tid] + red[3][tid]) / (float)K + eps);
    epi_sync();
  }
}

// Eight elements of HF's RMSNorm output: round(w * round(x * rstd)).
template <typename T>
__device__ __forceinline__ uint4 norm8(const uint4& xv, const uint4& wv, float rs) {
  float f[8], wf[8];
  Elem<T>::unpack(xv, f);
  Elem<T>::unpack(wv, wf);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    o[e] = pack2<T>(wf[2 * e] * round_to<T>(f[2 * e] * rs), wf[2 * e + 1] * round_to<T>(f[2 * e + 1] * rs));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int RP>
__device__ __forceinline__ void load_acc(uint32_t taddr, float* acc) {
  if constexpr (RP == 16) {
    tc::tmem_ld16(taddr, reinterpret_cast<uint32_t*>(acc));
  } else {
    tc::tmem_ld32(taddr, reinterpret_cast<uint32_t*>(acc));
  }
}

// Writes output feature `row` of tile t for every batch row.
template <typename T, int RP, int P>
__device__ __forceinline__ void store_tile(const LinearArgs& a, int t, int row, const float (&acc)[P][RP],
                                           float (&ssq)[RP], float (&yo)[RP], const float* rpre = nullptr) {
  int sj = 0, n;
  if constexpr (P == 2) {
    n = t * kTileN + row;
  } else {
    sj = seg_of_tile(a, t);
    n = (t - a.seg[sj].tile0) * kTileN + row;
  }
#pragma unroll
  for (int r = 0; r < RP; ++r) ssq[r] = yo[r] = 0.f;
  if (n >= a.seg[sj].rows) return;
  T* out = static_cast<T*>(a.seg[sj].out);
  const int64_t os = a.seg[sj].out_stride;
  const T* res = static_cast<const T*>(a.res);
  // every residual value is loaded before the first store: out may alias res,
  // which would otherwise serialise each load behind the previous store
  float rv[RP];
  if (P == 1 && a.mode == AICAS_LINEAR_RESIDUAL) {
#pragma unroll
    for (int r = 0; r < RP; ++r)
      if (r < a.R) rv[r] = rpre != nullptr ? rpre[r] : Elem<T>::to_float(res[r * a.res_stride + n]);
  }
#pragma unroll
  for (int r = 0; r < RP; ++r) {
    if (r < a.R) {
      float y;
      if constexpr (P == 2) {
        // HF Qwen3VLTextMLP: act_fn(gate_proj(x)) * up_proj(x), every product rounded to T
        const float g = round_to<T>(acc[0][r]);
        const float s = round_to<T>(g / (1.0f + expf(-g)));
        y = s * round_to<T>(acc[1][r]);
      } else {
        y = acc[0][r];
        if (a.mode == AICAS_LINEAR_RESIDUAL) y = rv[r] + round_to<T>(y);
      }
      const T yt = Elem<T>::from_float(y);
      out[r * os + n] = yt;
      const float yr = Elem<T>::to_float(yt);
      ssq[r] = yr * yr;
      yo[r] = yr;
    }
  }
}

template <typename T, int RP, int P>
__global__ void __launch_bounds__(kThreads, RP == 16 ? 2 : 1) decode_linear_kernel(const __grid_constant__ LinearArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_last;
  __shared__ float s_rstd[RP];
  __shared__ float s_red[4][8];
  __shared__ float s_red2[4][RP];

  constexpr uint32_t kCols = (2 * P * RP <= 32) ? 32u : (2 * P * RP <= 64 ? 64u : 128u);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int S = a.stages;
  const uint32_t ring = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t xs = ring + (uint32_t)(S * P * kTileBytes);
  const uint32_t recv = xs + (uint32_t)(a.n_slots * RP * 128);
  const uint32_t bars = recv + (uint32_t)a.recv_bytes;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (S + s); };
  auto accf = [&](int b) { return bars + 8u * (2 * S + b); };
  auto acce = [&](int b) { return bars + 8u * (2 * S + 2 + b); };
  const uint32_t xready = bars + 8u * (2 * S + 4);
  const uint32_t mdone = bars + 8u * (2 * S + 5);
  const uint32_t xload = bars + 8u * (2 * S + 6);  // x by TMA, before the in-place normalisation

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  // cluster split: tile c / cs, K blocks [q KB / cs, (q + 1) KB / cs) for rank q
  const int q_cl = a.cs > 0 ? c % a.cs : 0;
  const long long u0 = a.cs > 0 ? (long long)(c / a.cs) * a.KB + (long long)q_cl * a.KB / a.cs : unit_begin(a, c);
  const long long u1 =
      a.cs > 0 ? (long long)(c / a.cs) * a.KB + (long long)(q_cl + 1) * a.KB / a.cs : unit_begin(a, c + 1);
  const int n = (int)(u1 - u0);
  // the 64-K blocks this CTA reads, in X slots: all of them, or a contiguous run (mod KB)
  const int nfill = n < a.KB ? n : a.KB;
  const int kb0 = n < a.KB ? (int)(u0 % a.KB) : 0;
  volatile int* abort_flag = &s_abort;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf(b), 1);
      mbar_init(acce(b), kEpiThreads);
    }
    mbar_init(xready, 1);
    mbar_init(mdone, 1);
    mbar_init(xload, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tc::tmem_alloc(smem_u32(&s_tmem), kCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;
  const bool tmem_ok = (tmem >> 16) == 0 && (tmem & 0xFFFFu) % kCols == 0 && (tmem & 0xFFFFu) + kCols <= 512;
  if (!tmem_ok) {
    if (threadIdx.x == 0) flag_device_error(a.err, AICAS_DEVERR_TMEM);
  } else if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      for (int j = 0; j < a.nseg; ++j) tma_prefetch_desc(&a.seg[j].tm);
      if (a.x_tma) tma_prefetch_desc(&a.tm_x);
      const uint64_t pol = l2_policy_evict_first();
      auto issue = [&](int i) {
        const long long u = u0 + i;
        const int t = (int)(u / a.KB), kb = (int)(u % a.KB);
        const int s = i % S;
        mbar_arrive_expect_tx(full(s), P * kTileBytes);
#pragma unroll
        for (int p = 0; p < P; ++p) {
          int sj, row0;
          if constexpr (P == 2) {
            sj = p;
            row0 = t * kTileN;
          } else {
            sj = seg_of_tile(a, t);
            row0 = (t - a.seg[sj].tile0) * kTileN;
          }
          tma_load_2d_hint(ring + (uint32_t)((s * P + p) * kTileBytes), &a.seg[sj].tm, kb * kKBlock, row0, full(s),
                           pol);
        }
      };
      // the weights depend on nothing: fill the ring before waiting for the
      // previous kernel, then bring x' in as soon as it is complete
      const int pre = n < S ? n : S;
      for (int i = 0; i < pre; ++i) issue(i);
      int issued = pre;
      const int pf_end = n < pre + a.pf_units ? n : pre + a.pf_units;
      for (int i = pre; i < pf_end; ++i) {
        const long long u = u0 + i;
        const int t = (int)(u / a.KB), kb = (int)(u % a.KB);
#pragma unroll
        for (int p = 0; p < P; ++p) {
          int sj, row0;
          if constexpr (P == 2) {
            sj = p;
            row0 = t * kTileN;
          } else {
            sj = seg_of_tile(a, t);
            row0 = (t - a.seg[sj].tile0) * kTileN;
          }
          tma_prefetch_l2_2d(&a.seg[sj].tm, kb * kKBlock, row0);
        }
      }
      if (a.x_tma) {
        grid_dependency_wait();
        const uint64_t keep = l2_policy_evict_last();
        const uint32_t xbar = a.norm_w != nullptr ? xload : xready;
        mbar_arrive_expect_tx(xbar, (uint32_t)(nfill * RP * 128));
        for (int j = 0; j < nfill; ++j)
          tma_load_2d_hint(xs + (uint32_t)(j * RP * 128), &a.tm_x, ((kb0 + j) % a.KB) * kKBlock, 0, xbar, keep);
      }
      for (int i = pre; i < n; ++i) {
        if (!mbar_wait(empty(i % S), ((i / S) - 1) & 1, abort_flag, a.err)) break;
        issue(i);
        issued = i + 1;
      }
      // every copy issued lands before the CTA can exit (the last one per stage, and x')
      for (int i = issued > S ? issued - S : 0; i < issued; ++i) mbar_wait(full(i % S), (i / S) & 1, nullptr, a.err);
      if (a.x_tma) mbar_wait(a.norm_w != nullptr ? xload : xready, 0, nullptr, a.err);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = tc::idesc_f16(kBf16, kTileN, RP, false, false);
      bool ok = mbar_wait(xready, 0, abort_flag, a.err);
      int portion = 0;
      for (int i = 0; ok && i < n; ++i) {
        const long long u = u0 + i;
        const int kb = (int)(u % a.KB);
        const int s = i % S;
        const bool first = i == 0 || kb == 0;
        const bool last = i == n - 1 || kb == a.KB - 1;
        const int buf = portion & 1;
        if (first && portion >= 2 && !mbar_wait(acce(buf), ((portion >> 1) - 1) & 1, abort_flag, a.err)) break;
        if (!mbar_wait(full(s), (i / S) & 1, abort_flag, a.err)) break;
        tc::fence_after_sync();
        const int slot = (kb - kb0 + a.KB) % a.KB;
        const uint64_t bdesc = tc::smem_desc_sw128(xs + (uint32_t)(slot * RP * 128), 16, 1024);
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const uint64_t adesc = tc::smem_desc_sw128(ring + (uint32_t)((s * P + p) * kTileBytes), 16, 1024);
          const uint32_t d = tmem + (uint32_t)(buf * P * RP + p * RP);
#pragma unroll
          for (int ks = 0; ks < kKBlock / 16; ++ks)
            tc::mma_f16_ss(d, adesc + 2 * ks, bdesc + 2 * ks, idesc, (first && ks == 0) ? 0u : 1u);
        }
        tc::commit(empty(s));
        if (last) {
          tc::commit(accf(buf));
          ++portion;
        }
      }
      // the next kernel's CTAs (and their weight traffic) may start once this
      // CTA has issued its last product: earlier, their L2 prefetch slows this
      // kernel's own epilogue loads (measured)
      grid_launch_dependents();
      // every product issued has completed before TMEM is released
      tc::commit(mdone);
      mbar_wait(mdone, 0, nullptr, a.err);
    }
  } else {
    // ------------------------------------------------------------ prologue + epilogue
    const int tid = threadIdx.x;  // 0..127 = TMEM lane = feature within the tile
    const T* x = static_cast<const T*>(a.x);
    const T* nw = static_cast<const T*>(a.norm_w);
    // the norm weights depend on nothing: fetched while the previous kernel
    // finishes.  Thread tid normalises the (slot, 16-byte chunk) pairs tid,
    // tid + 128, ... of x in place; the first kNormPre pairs' weights are kept.
    constexpr int kNormPre = 4;
    const bool norm_in_place = a.x_tma && nw != nullptr;
    uint4 wpre[kNormPre];
    if (norm_in_place) {
#pragma unroll
      for (int m = 0; m < kNormPre; ++m) {
        const int pair = tid + m * kEpiThreads;
        const int k = ((kb0 + (pair >> 3)) % a.KB) * kKBlock + (pair & 7) * 8;
        if (pair < nfill * 8 && k < a.K) wpre[m] = *reinterpret_cast<const uint4*>(nw + k);
      }
    }
    grid_dependency_wait();
    // cluster split with a residual: the owner's residual values, loaded now
    // rather than behind the reduction
    const int fs_own = a.cs > 1 ? (kTileN + a.cs - 1) / a.cs : kTileN;
    float rpre[RP];
    const bool res_pre = P == 1 && a.cs > 1 && a.mode == AICAS_LINEAR_RESIDUAL && tid < fs_own &&
                         q_cl * fs_own + tid < kTileN && (c / a.cs) * kTileN + q_cl * fs_own + tid < a.seg[0].rows;
    if (res_pre) {
      const int n_own = (c / a.cs) * kTileN + q_cl * fs_own + tid;
      const T* res = static_cast<const T*>(a.res);
#pragma unroll
      for (int r = 0; r < RP; ++r)
        if (r < a.R) rpre[r] = Elem<T>::to_float(res[r * a.res_stride + n_own]);
    }
    if (!a.x_tma) {
      if (nw != nullptr) block_rstd<T, false>(x, a.x_stride, a.R, a.K, a.eps, s_rstd, s_red);
      // X' into the slots: [RP rows x 64] per K block, 128-byte rows, 16-byte
      // chunks swizzled by row (the layout TMA gives a 128B-swizzled box).  The
      // real rows first, eight loads in flight per thread; then zeros in the
      // padding rows.
      const int items = nfill * a.R * 8;
      for (int base = tid; base < items; base += 8 * kEpiThreads) {
        uint4 v[8], w[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int idx = base + m * kEpiThreads;
          if (idx < items) {
            const int j = idx / (a.R * 8), rem = idx % (a.R * 8), r = rem >> 3, ch = rem & 7;
            const int k = ((kb0 + j) % a.KB) * kKBlock + ch * 8;
            v[m] = make_uint4(0u, 0u, 0u, 0u);
            if (k < a.K) {
              v[m] = *reinterpret_cast<const uint4*>(x + r * a.x_stride + k);
              if (nw != nullptr) w[m] = *reinterpret_cast<const uint4*>(nw + k);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int idx = base + m * kEpiThreads;
          if (idx < items) {
            const int j = idx / (a.R * 8), rem = idx % (a.R * 8), r = rem >> 3, ch = rem & 7;
            const int k = ((kb0 + j) % a.KB) * kKBlock + ch * 8;
            const uint4 o4 = (nw != nullptr && k < a.K) ? norm8<T>(v[m], w[m], s_rstd[r]) : v[m];
            const uint32_t dst = xs + (uint32_t)(j * RP * 128 + r * 128 + ((ch ^ (r & 7)) << 4));
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(o4.x), "r"(o4.y), "r"(o4.z),
                         "r"(o4.w)
                         : "memory");
          }
        }
      }
      const int pad_items = nfill * (RP - a.R) * 8;
      for (int idx = tid; idx < pad_items; idx += kEpiThreads) {
        const int j = idx / ((RP - a.R) * 8), rem = idx % ((RP - a.R) * 8), r = a.R + (rem >> 3), ch = rem & 7;
        const uint32_t dst = xs + (uint32_t)(j * RP * 128 + r * 128 + ((ch ^ (r & 7)) << 4));
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
      }
      fence_proxy_async_smem();
      epi_sync();
      if (tid == 0) mbar_arrive(xready);
    } else if (nw != nullptr) {
      // x arrived by TMA; its RMSNorm statistics come with it (x_sumsq): the
      // normalisation runs on the slots in place, rounded as HF rounds
      if (tid < a.R) s_rstd[tid] = rsqrtf(a.x_sumsq[tid] / (float)a.K + a.eps);
      const bool landed = epi_all(mbar_wait(xload, 0, abort_flag, a.err));
      if (landed) {
        const int pairs = nfill * 8;
        for (int pair = tid, m = 0; pair < pairs; pair += kEpiThreads, ++m) {
          const int j = pair >> 3, ch = pair & 7;
          const int k = ((kb0 + j) % a.KB) * kKBlock + ch * 8;
          if (k >= a.K) continue;
          uint4 w;
          if (m < kNormPre) {
#pragma unroll
            for (int q = 0; q < kNormPre; ++q)
              if (q == m) w = wpre[q];
          } else {
            w = *reinterpret_cast<const uint4*>(nw + k);
          }
          for (int r = 0; r < a.R; ++r) {
            const uint32_t at = xs + (uint32_t)(j * RP * 128 + r * 128 + ((ch ^ (r & 7)) << 4));
            uint4 v;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"(at));
            const uint4 o4 = norm8<T>(v, w, s_rstd[r]);
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(at), "r"(o4.x), "r"(o4.y), "r"(o4.z),
                         "r"(o4.w)
                         : "memory");
          }
        }
        fence_proxy_async_smem();
      }
      epi_sync();
      if (tid == 0 && landed) mbar_arrive(xready);
    }

    int portion = 0;
    bool aborted = false;
    float ssq[RP], yo[RP];
    const int fs = a.cs > 1 ? (kTileN + a.cs - 1) / a.cs : kTileN;  // cluster split: features per rank
    if (a.cs > 1) {
      // ---- cluster split: one tile per cluster, each rank's partial row goes
      // to the rank that owns its feature; the owners add them in rank order
      const int t = c / a.cs;
      const bool got = mbar_wait(accf(0), 0, abort_flag, a.err);
      aborted = !epi_all(got);
      if (!aborted) {
        tc::fence_after_sync();
        float acc[P][RP];
        const uint32_t lanes = (uint32_t)(warp * 32) << 16;
#pragma unroll
        for (int p = 0; p < P; ++p) load_acc<RP>(tmem + lanes + (uint32_t)(p * RP), acc[p]);
        tc::tmem_wait_ld();
        tc::fence_before_sync();
        mbar_arrive(acce(0));
        const int j = tid / fs, l = tid % fs;
        const uint32_t dst = cluster_map(recv + (uint32_t)((q_cl * fs + l) * P * RP * 4), (uint32_t)j);
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
          for (int r = 0; r < RP; r += 4)
            st_cluster_v4(dst + (uint32_t)((p * RP + r) * 4), acc[p][r], acc[p][r + 1], acc[p][r + 2], acc[p][r + 3]);
      }
      __syncwarp();
      cluster_sync_all();
#pragma unroll
      for (int r = 0; r < RP; ++r) ssq[r] = yo[r] = 0.f;
      const int row = q_cl * fs + tid;
      if (!aborted && tid < fs && row < kTileN) {
        float sum[P][RP];
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
          for (int r = 0; r < RP; ++r) sum[p][r] = 0.f;
        for (int q = 0; q < a.cs; ++q) {
          const uint32_t src = recv + (uint32_t)((q * fs + tid) * P * RP * 4);
#pragma unroll
          for (int p = 0; p < P; ++p)
#pragma unroll
            for (int r = 0; r < RP; r += 4) {
              float4 v;
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                           : "r"(src + (uint32_t)((p * RP + r) * 4)));
              sum[p][r] += v.x;
              sum[p][r + 1] += v.y;
              sum[p][r + 2] += v.z;
              sum[p][r + 3] += v.w;
            }
        }
        store_tile<T, RP, P>(a, t, row, sum, ssq, yo, res_pre ? rpre : nullptr);
      }
      if (a.sumsq_out != nullptr && !aborted) {
        // this slice's share of the next RMSNorm: per-row sums of squares
#pragma unroll
        for (int r = 0; r < RP; ++r) {
          if (r < a.R) {
            float v = ssq[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) s_red2[warp][r] = v;
          }
        }
        epi_sync();
        if (tid < a.R) a.ss_part[c * RP + tid] = s_red2[0][tid] + s_red2[1][tid] + s_red2[2][tid] + s_red2[3][tid];
        epi_sync();
      }
    }
    for (long long u = a.cs > 1 ? u1 : u0; u < u1;) {
      const int t = (int)(u / a.KB);
      const long long tile_end = (long long)(t + 1) * a.KB;
      const int buf = portion & 1;
      const bool got = mbar_wait(accf(buf), (portion >> 1) & 1, abort_flag, a.err);
      if (!epi_all(got)) {
        aborted = true;
        break;
      }
      tc::fence_after_sync();
      float acc[P][RP];
      const uint32_t lanes = (uint32_t)(warp * 32) << 16;
#pragma unroll
      for (int p = 0; p < P; ++p) load_acc<RP>(tmem + lanes + (uint32_t)(buf * P * RP + p * RP), acc[p]);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      mbar_arrive(acce(buf));
      ++portion;
      const int cf = cta_of_unit(a, (long long)t * a.KB), cl = cta_of_unit(a, tile_end - 1);
      u = tile_end < u1 ? tile_end : u1;
      if (cf != cl) {
        // shared tile: publish this CTA's partial; the last contributor adds them up
        float* mine = a.partials + (size_t)partial_slot(a, c, t) * (P * RP * kTileN);
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
          for (int r = 0; r < RP; ++r)
            if (r < a.R) mine[(p * RP + r) * kTileN + tid] = acc[p][r];
        // the barrier orders every thread's stores before thread 0's release
        // (cumulative): one fence for the CTA, in the atomic
        epi_sync();
        if (tid == 0) {
          const unsigned int old = atom_add_acq_rel(a.counters + t, 1u);
          const int last = old == (unsigned int)(cl - cf);
          if (last) a.counters[t] = 0u;
          s_last = last;
        }
        epi_sync();
        if (!s_last) continue;
        fence_acq_rel_gpu();
        // add the partials in CTA order, G contributors' loads in flight at once
        constexpr int G = (P * RP <= 16) ? 2 : 1;
        float sum[P][RP];
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
          for (int r = 0; r < RP; ++r) sum[p][r] = 0.f;
        for (int cc0 = cf; cc0 <= cl; cc0 += G) {
          float v[G][P][RP];
#pragma unroll
          for (int q = 0; q < G; ++q) {
            const int cc = cc0 + q;
            if (cc <= cl && cc != c) {
              const float* src = a.partials + (size_t)partial_slot(a, cc, t) * (P * RP * kTileN);
#pragma unroll
              for (int p = 0; p < P; ++p)
#pragma unroll
                for (int r = 0; r < RP; ++r)
                  if (r < a.R) v[q][p][r] = __ldcg(src + (p * RP + r) * kTileN + tid);
            }
          }
#pragma unroll
          for (int q = 0; q < G; ++q) {
            const int cc = cc0 + q;
            if (cc <= cl) {
#pragma unroll
              for (int p = 0; p < P; ++p)
#pragma unroll
                for (int r = 0; r < RP; ++r) sum[p][r] += cc == c ? acc[p][r] : v[q][p][r];
            }
          }
        }
        store_tile<T, RP, P>(a, t, tid, sum, ssq, yo);
      } else {
        store_tile<T, RP, P>(a, t, tid, acc, ssq, yo);
      }
      if (a.sumsq_out != nullptr) {
        // this tile's share of the next RMSNorm: per-row sums of squares
#pragma unroll
        for (int r = 0; r < RP; ++r) {
          if (r < a.R) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ssq[r] += __shfl_xor_sync(0xffffffffu, ssq[r], o);
            if (lane == 0) s_red2[warp][r] = ssq[r];
          }
        }
        epi_sync();
        if (tid < a.R) a.ss_part[t * RP + tid] = s_red2[0][tid] + s_red2[1][tid] + s_red2[2][tid] + s_red2[3][tid];
        epi_sync();
      }
    }
    if (a.sumsq_out != nullptr && !aborted) {
      // the last CTA to finish adds the shares up in a fixed order (the
      // barrier orders the shares' stores before thread 0's release)
      epi_sync();
      if (tid == 0) {
        const unsigned int old = atom_add_acq_rel(a.counters + kDoneSlot, 1u);
        const int last = old == (unsigned int)(a.grid - 1);
        if (last) a.counters[kDoneSlot] = 0u;
        s_last = last;
      }
      epi_sync();
      if (s_last) {
        // a fixed order, in parallel: kTpr consecutive lanes per row each add
        // every kTpr-th share (eight loads in flight), then a butterfly over
        // those lanes
        fence_acq_rel_gpu();
        constexpr int kTpr = kEpiThreads / RP;  // 8 or 4 lanes of one warp per row
        const int count = a.cs > 1 ? a.grid : a.tiles;
        const int r = tid / kTpr, j = tid % kTpr;
        float ss = 0.f;
        if (r < a.R) {
          for (int e0 = j; e0 < count; e0 += 8 * kTpr) {
            float v[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
              const int e = e0 + m * kTpr;
              v[m] = e < count ? __ldcg(a.ss_part + e * RP + r) : 0.f;
            }
#pragma unroll
            for (int m = 0; m < 8; ++m) ss += v[m];
          }
        }
#pragma unroll
        for (int o = kTpr / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (j == 0 && r < a.R) a.sumsq_out[r] = ss;
      }
    }
  }

  if (a.cs > 1 && (!tmem_ok || warp >= 4)) {
    __syncwarp();
    cluster_sync_all();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kCols);
  }
}

// ------------------------------------------------------------------ host side

struct Plan {
  int RP, P, tiles, KB, grid, stages, n_slots, cs, recv_bytes;
  long long units;
  size_t counter_bytes, partial_bytes, ss_bytes, smem;
  int pf_units;
};

int tiles_of(int rows) { return (rows + kTileN - 1) / kTileN; }

int make_plan(const aicas_linear_params* p, int sms, Plan* pl, char* err, size_t errlen) {
  pl->RP = p->batch <= 16 ? 16 : 32;
  pl->P = p->mode == AICAS_LINEAR_SWIGLU ? 2 : 1;
  pl->KB = (p->in_features + kKBlock - 1) / kKBlock;
  int tiles = 0;
  if (pl->P == 2) {
    tiles = tiles_of(p->seg[0].rows);
  } else {
    for (int j = 0; j < p->num_segments; ++j) tiles += tiles_of(p->seg[j].rows);
  }
  if (tiles > kMaxTiles) {
    snprintf(err, errlen, "decode linear: %d output tiles of %d features exceed the %d the workspace counts", tiles,
             kTileN, kMaxTiles);
    return AICAS_ERR_UNSUPPORTED;
  }
  pl->tiles = tiles;
  pl->units = (long long)tiles * pl->KB;
  // fewer tiles than SMs: a cluster of cs CTAs per tile splits K and adds the
  // partials through distributed shared memory; otherwise stream-K ranges
  pl->cs = 0;
  if (tiles < sms && (p->flags & AICAS_LINEAR_STREAM_K) == 0) {
    int cs = sms / tiles;
    if (cs > 8) cs = 8;
    if (cs > pl->KB) cs = pl->KB;
    pl->cs = cs < 1 ? 1 : cs;
  }
  int grid = pl->cs > 0 ? tiles * pl->cs : (int)(pl->units < sms ? pl->units : sms);
  pl->recv_bytes = 0;
  if (pl->cs > 1) {
    const int fs = (kTileN + pl->cs - 1) / pl->cs;
    pl->recv_bytes = pl->cs * fs * pl->P * pl->RP * 4;
  }
  const size_t bar_bytes = 8 * (2 * kMaxStages + 7);
  for (;;) {
    const long long per = pl->cs > 0 ? (pl->KB + pl->cs - 1) / pl->cs : (pl->units + grid - 1) / grid;
    pl->n_slots = (int)(per < pl->KB ? per : pl->KB);
    const long long x_bytes = (long long)pl->n_slots * pl->RP * 128 + pl->recv_bytes;
    const int cap = kMaxStages / pl->P;
    // two CTAs per SM while that leaves 64 KB of stages (the next product's
    // CTAs then fill their rings during this one); a whole SM otherwise.  (A
    // whole SM for the paired gate/up tiles measured slower: its clusters of
    // three no longer all fit at once beside the previous product's CTAs.)
    const long long room2 = kSmemTwoPerSm - 1024 - (long long)bar_bytes - x_bytes;
    int stages = room2 > 0 ? (int)(room2 / ((long long)pl->P * kTileBytes)) : 0;
    if (stages * pl->P < 4) {
      const long long room = kSmemBudget - 1024 - (long long)bar_bytes - x_bytes;
      stages = room > 0 ? (int)(room / ((long long)pl->P * kTileBytes)) : 0;
    }
    if (stages > cap) stages = cap;
    if (stages >= 2) {
      pl->stages = stages;
      pl->smem = 1024 + (size_t)stages * pl->P * kTileBytes + (size_t)x_bytes + bar_bytes;
      break;
    }
    if (pl->cs > 0 || grid >= pl->units) {
      snprintf(err, errlen, "decode linear: in_features=%d with %d rows does not fit shared memory", p->in_features,
               p->batch);
      return AICAS_ERR_UNSUPPORTED;
    }
    grid = (int)(2LL * grid < pl->units ? 2LL * grid : pl->units);
  }
  pl->grid = grid;
  pl->counter_bytes = kCounterRegion;
  pl->partial_bytes = pl->cs > 0 ? 0 : (size_t)2 * grid * pl->P * pl->RP * kTileN * 4;
  const int shares = pl->cs > 1 ? grid : tiles;
  pl->ss_bytes = p->sumsq_out != nullptr ? ((size_t)shares * pl->RP * 4 + 255) / 256 * 256 : 0;
  {
    const long long per = pl->cs > 0 ? (pl->KB + pl->cs - 1) / pl->cs : (pl->units + grid - 1) / grid;
    long long cap = kL2PrefetchBytes / ((long long)grid * pl->P * kTileBytes);
    pl->pf_units = (int)(per < cap ? per : cap);
  }
  return AICAS_OK;
}

bool make_weight_map(CUtensorMap* m, const aicas_linear_segment& s, int K, bool bf16, char* err, size_t errlen) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (enc == nullptr) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)s.rows};
  cuuint64_t strides[1] = {(cuuint64_t)s.weight_stride * 2};
  cuuint32_t box[2] = {kKBlock, kTileN};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(s.weight), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (%d) for a [%d, %d] weight with row stride %lld", (int)r,
             s.rows, K, (long long)s.weight_stride);
    return false;
  }
  return true;
}

// x' [R, K] with rows RP apart in the box: rows past R are read as zeros.
bool make_x_map(CUtensorMap* m, const void* x, int64_t stride, int R, int K, int RP, bool bf16, char* err,
                size_t errlen) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (enc == nullptr) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)R};
  cuuint64_t strides[1] = {(cuuint64_t)(R > 1 ? stride : K) * 2};
  cuuint32_t box[2] = {kKBlock, (cuuint32_t)RP};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (%d) for x [%d, %d] with row stride %lld", (int)r, R, K,
             (long long)stride);
    return false;
  }
  return true;
}

template <typename T, int RP, int P>
cudaError_t launch_t(const LinearArgs& a, size_t smem, bool pdl, cudaStream_t st) {
  // (cluster split when a.cs > 1: one cluster of a.cs CTAs per tile)
  auto kern = decode_linear_kernel<T, RP, P>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)a.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (a.cs > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)a.cs;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename T>
cudaError_t dispatch(const LinearArgs& a, const Plan& pl, bool pdl, cudaStream_t st) {
  if (pl.RP == 16) {
    return pl.P == 2 ? launch_t<T, 16, 2>(a, pl.smem, pdl, st) : launch_t<T, 16, 1>(a, pl.smem, pdl, st);
  }
  return pl.P == 2 ? launch_t<T, 32, 2>(a, pl.smem, pdl, st) : launch_t<T, 32, 1>(a, pl.smem, pdl, st);
}

}  // namespace

int plan_linear_workspace(const aicas_linear_params* p, int sms, size_t* bytes, char* err, size_t errlen) {
  *bytes = 0;
  if (p->batch == 0) return AICAS_OK;
  Plan pl;
  const int rc = make_plan(p, sms, &pl, err, errlen);
  if (rc != AICAS_OK) return rc;
  *bytes = pl.counter_bytes + pl.partial_bytes + pl.ss_bytes;
  return AICAS_OK;
}

int run_linear(const aicas_linear_params* p, int sms, void* workspace, size_t workspace_bytes, cudaStream_t stream,
               unsigned int* dev_err, char* err, size_t errlen) {
  if (p->batch == 0) return AICAS_OK;
  Plan pl;
  int rc = make_plan(p, sms, &pl, err, errlen);
  if (rc != AICAS_OK) return rc;
  const size_t need = pl.counter_bytes + pl.partial_bytes + pl.ss_bytes;
  if (workspace == nullptr || workspace_bytes < need) {
    snprintf(err, errlen, "decode linear needs %zu bytes of zero-initialised workspace (got %zu)", need,
             workspace == nullptr ? (size_t)0 : workspace_bytes);
    return AICAS_ERR_WORKSPACE;
  }
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
    snprintf(err, errlen, "workspace must be 256-byte aligned");
    return AICAS_ERR_INVALID;
  }
  const bool bf16 = p->dtype == AICAS_DTYPE_BF16;
  LinearArgs a;
  memset(&a, 0, sizeof(a));
  int tile0 = 0;
  for (int j = 0; j < p->num_segments; ++j) {
    if (!make_weight_map(&a.seg[j].tm, p->seg[j], p->in_features, bf16, err, errlen)) return AICAS_ERR_UNSUPPORTED;
    a.seg[j].out = p->seg[j].out;
    a.seg[j].out_stride = p->seg[j].out_stride;
    a.seg[j].rows = p->seg[j].rows;
    a.seg[j].tile0 = pl.P == 2 ? 0 : tile0;
    tile0 += tiles_of(p->seg[j].rows);
  }
  a.x_tma = (p->norm_weight == nullptr || p->x_sumsq != nullptr) ? 1 : 0;
  if (a.x_tma && !make_x_map(&a.tm_x, p->x, p->x_stride, p->batch, p->in_features, pl.RP, bf16, err, errlen))
    return AICAS_ERR_UNSUPPORTED;
  a.sumsq_out = p->sumsq_out;
  a.x_sumsq = p->x_sumsq;
  a.x = p->x;
  a.x_stride = p->x_stride;
  a.norm_w = p->norm_weight;
  a.res = p->residual;
  a.res_stride = p->residual_stride;
  a.eps = p->eps;
  a.R = p->batch;
  a.K = p->in_features;
  a.KB = pl.KB;
  a.nseg = p->num_segments;
  a.mode = p->mode;
  a.tiles = pl.tiles;
  a.grid = pl.grid;
  a.stages = pl.stages;
  a.n_slots = pl.n_slots;
  a.units = pl.units;
  a.counters = static_cast<uint32_t*>(workspace);
  a.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + pl.counter_bytes);
  a.ss_part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + pl.counter_bytes + pl.partial_bytes);
  a.pf_units = pl.pf_units;
  a.cs = pl.cs;
  a.recv_bytes = pl.recv_bytes;
  a.err = dev_err;
  const bool pdl = (p->flags & AICAS_LINEAR_NO_PDL) == 0;
  const cudaError_t e = bf16 ? dispatch<__nv_bfloat16>(a, pl, pdl, stream) : dispatch<__half>(a, pl, pdl, stream);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "decode linear launch: %s (%s)", cudaGetErrorString(e), cudaGetErrorName(e));
    return AICAS_ERR_CUDA;
  }
  return AICAS_OK;
}

}  // namespace aicas
