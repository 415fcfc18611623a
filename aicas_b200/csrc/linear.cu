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
// epilogue (activations, outputs, workspace) wait for it.
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
constexpr int kMaxStages = 8;
// The tile counters sit in a fixed region at the start of every workspace, so
// calls of different shapes can share one workspace: a call's partials never
// land on another call's counters.
constexpr size_t kCounterRegion = 64 << 10;
constexpr int kMaxTiles = (int)(kCounterRegion / 4);

struct LinSeg {
  CUtensorMap tm;  // 2-D [rows, K], box {64, 128}, 128-byte swizzle
  void* out;
  int64_t out_stride;
  int rows;
  int tile0;  // first tile index of the segment
};

struct LinearArgs {
  LinSeg seg[AICAS_LINEAR_MAX_SEGMENTS];
  const void* x;
  int64_t x_stride;
  const void* norm_w;
  const void* res;
  int64_t res_stride;
  float eps;
  int R, K, KB, nseg, mode, tiles, grid, stages, n_slots;
  long long units;
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
__device__ __forceinline__ void store_tile(const LinearArgs& a, int t, int row, const float (&acc)[P][RP]) {
  int sj = 0, n;
  if constexpr (P == 2) {
    n = t * kTileN + row;
  } else {
    sj = seg_of_tile(a, t);
    n = (t - a.seg[sj].tile0) * kTileN + row;
  }
  if (n >= a.seg[sj].rows) return;
  T* out = static_cast<T*>(a.seg[sj].out);
  const int64_t os = a.seg[sj].out_stride;
  const T* res = static_cast<const T*>(a.res);
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
        if (a.mode == AICAS_LINEAR_RESIDUAL) y = Elem<T>::to_float(res[r * a.res_stride + n]) + round_to<T>(y);
      }
      out[r * os + n] = Elem<T>::from_float(y);
    }
  }
}

template <typename T, int RP, int P>
__global__ void __launch_bounds__(kThreads, 1) decode_linear_kernel(const __grid_constant__ LinearArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_last;
  __shared__ float s_rstd[RP];

  constexpr uint32_t kCols = (2 * P * RP <= 32) ? 32u : (2 * P * RP <= 64 ? 64u : 128u);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int S = a.stages;
  const uint32_t ring = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t xs = ring + (uint32_t)(S * P * kTileBytes);
  const uint32_t bars = xs + (uint32_t)(a.n_slots * RP * 128);
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (S + s); };
  auto accf = [&](int b) { return bars + 8u * (2 * S + b); };
  auto acce = [&](int b) { return bars + 8u * (2 * S + 2 + b); };
  const uint32_t xready = bars + 8u * (2 * S + 4);
  const uint32_t mdone = bars + 8u * (2 * S + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = unit_begin(a, c), u1 = unit_begin(a, c + 1);
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
  if (threadIdx.x == 0) grid_launch_dependents();
  const bool tmem_ok = (tmem >> 16) == 0 && (tmem & 0xFFFFu) % kCols == 0 && (tmem & 0xFFFFu) + kCols <= 512;
  if (!tmem_ok) {
    if (threadIdx.x == 0) flag_device_error(a.err, AICAS_DEVERR_TMEM);
  } else if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      for (int j = 0; j < a.nseg; ++j) tma_prefetch_desc(&a.seg[j].tm);
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const long long u = u0 + i;
        const int t = (int)(u / a.KB), kb = (int)(u % a.KB);
        const int s = i % S;
        if (i >= S && !mbar_wait(empty(s), ((i / S) - 1) & 1, abort_flag, a.err)) break;
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
        issued = i + 1;
      }
      // every copy issued lands before the CTA can exit (the last one per stage)
      for (int i = issued > S ? issued - S : 0; i < issued; ++i) mbar_wait(full(i % S), (i / S) & 1, nullptr, a.err);
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
      // every product issued has completed before TMEM is released
      tc::commit(mdone);
      mbar_wait(mdone, 0, nullptr, a.err);
    }
  } else {
    // ------------------------------------------------------------ prologue + epilogue
    const int tid = threadIdx.x;  // 0..127 = TMEM lane = feature within the tile
    grid_dependency_wait();
    const T* x = static_cast<const T*>(a.x);
    const T* nw = static_cast<const T*>(a.norm_w);
    if (nw != nullptr) {
      // HF Qwen3VLTextRMSNorm statistics: mean of squares in fp32
      for (int r = warp; r < a.R; r += 4) {
        const T* xr = x + r * a.x_stride;
        float ss = 0.f;
        for (int k = lane * 8; k < a.K; k += 256) {
          float f[8];
          Elem<T>::unpack(*reinterpret_cast<const uint4*>(xr + k), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) s_rstd[r] = rsqrtf(ss / (float)a.K + a.eps);
      }
      epi_sync();
    }
    // X' into the slots: [RP rows x 64] per K block, 128-byte rows, 16-byte
    // chunks swizzled by row (the layout TMA gives a 128B-swizzled box)
    for (int idx = tid; idx < nfill * RP * 8; idx += kEpiThreads) {
      const int j = idx / (RP * 8), rem = idx % (RP * 8), r = rem >> 3, ch = rem & 7;
      const int k = ((kb0 + j) % a.KB) * kKBlock + ch * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < a.R && k < a.K) {
        v = *reinterpret_cast<const uint4*>(x + r * a.x_stride + k);
        if (nw != nullptr) {
          float f[8], w[8];
          Elem<T>::unpack(v, f);
          Elem<T>::unpack(*reinterpret_cast<const uint4*>(nw + k), w);
          const float rs = s_rstd[r];
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            o[e] = pack2<T>(w[2 * e] * round_to<T>(f[2 * e] * rs), w[2 * e + 1] * round_to<T>(f[2 * e + 1] * rs));
          v = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      const uint32_t dst = xs + (uint32_t)(j * RP * 128 + r * 128 + ((ch ^ (r & 7)) << 4));
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                   : "memory");
    }
    fence_proxy_async_smem();
    epi_sync();
    if (tid == 0) mbar_arrive(xready);

    int portion = 0;
    for (long long u = u0; u < u1;) {
      const int t = (int)(u / a.KB);
      const long long tile_end = (long long)(t + 1) * a.KB;
      const int buf = portion & 1;
      const bool got = mbar_wait(accf(buf), (portion >> 1) & 1, abort_flag, a.err);
      if (!epi_all(got)) break;
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
        __threadfence();
        epi_sync();
        if (tid == 0) {
          const unsigned int old = atom_add_acq_rel(a.counters + t, 1u);
          const int last = old == (unsigned int)(cl - cf);
          if (last) a.counters[t] = 0u;
          s_last = last;
        }
        epi_sync();
        if (!s_last) continue;
        __threadfence();
        float sum[P][RP];
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
          for (int r = 0; r < RP; ++r) sum[p][r] = 0.f;
        for (int cc = cf; cc <= cl; ++cc) {
          if (cc == c) {
#pragma unroll
            for (int p = 0; p < P; ++p)
#pragma unroll
              for (int r = 0; r < RP; ++r) sum[p][r] += acc[p][r];
          } else {
            const float* q = a.partials + (size_t)partial_slot(a, cc, t) * (P * RP * kTileN);
#pragma unroll
            for (int p = 0; p < P; ++p)
#pragma unroll
              for (int r = 0; r < RP; ++r)
                if (r < a.R) sum[p][r] += __ldcg(q + (p * RP + r) * kTileN + tid);
          }
        }
        store_tile<T, RP, P>(a, t, tid, sum);
      } else {
        store_tile<T, RP, P>(a, t, tid, acc);
      }
    }
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
  int RP, P, tiles, KB, grid, stages, n_slots;
  long long units;
  size_t counter_bytes, partial_bytes, smem;
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
  int grid = (int)(pl->units < sms ? pl->units : sms);
  const size_t bar_bytes = 8 * (2 * kMaxStages + 6);
  for (;;) {
    const long long per = (pl->units + grid - 1) / grid;
    pl->n_slots = (int)(per < pl->KB ? per : pl->KB);
    const long long x_bytes = (long long)pl->n_slots * pl->RP * 128;
    const long long room = kSmemBudget - 1024 - (long long)bar_bytes - x_bytes;
    int stages = room > 0 ? (int)(room / ((long long)pl->P * kTileBytes)) : 0;
    const int cap = kMaxStages / pl->P;
    if (stages > cap) stages = cap;
    if (stages >= 2) {
      pl->stages = stages;
      pl->smem = 1024 + (size_t)stages * pl->P * kTileBytes + (size_t)x_bytes + bar_bytes;
      break;
    }
    if (grid >= pl->units) {
      snprintf(err, errlen, "decode linear: in_features=%d with %d rows does not fit shared memory", p->in_features,
               p->batch);
      return AICAS_ERR_UNSUPPORTED;
    }
    grid = (int)(2LL * grid < pl->units ? 2LL * grid : pl->units);
  }
  pl->grid = grid;
  pl->counter_bytes = kCounterRegion;
  pl->partial_bytes = (size_t)2 * grid * pl->P * pl->RP * kTileN * 4;
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

template <typename T, int RP, int P>
cudaError_t launch_t(const LinearArgs& a, size_t smem, bool pdl, cudaStream_t st) {
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
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
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
  *bytes = pl.counter_bytes + pl.partial_bytes;
  return AICAS_OK;
}

int run_linear(const aicas_linear_params* p, int sms, void* workspace, size_t workspace_bytes, cudaStream_t stream,
               unsigned int* dev_err, char* err, size_t errlen) {
  if (p->batch == 0) return AICAS_OK;
  Plan pl;
  int rc = make_plan(p, sms, &pl, err, errlen);
  if (rc != AICAS_OK) return rc;
  const size_t need = pl.counter_bytes + pl.partial_bytes;
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
