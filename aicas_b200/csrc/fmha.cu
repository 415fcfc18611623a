// Flash-attention forward on the sm_100a tensor cores: causal GQA prefill and
// non-causal packed-varlen (ViT) attention.
//
// Replaces the reference's Triton kernels
//   triton_qwen3vl/gqa_flash_attention.py:79-190   (_gqa_flash_attention_fwd)
//   triton_qwen3vl/varlen_flash_attention.py:149-264 (_varlen_flash_attention_fwd)
// with the same math: S = Q K^T, online softmax in base 2 with fp32 statistics,
// P rounded to the input dtype before P V (gqa_flash_attention.py:178), O / l.
//
// One CTA owns two 128-row query tiles that read the SAME key/value head:
// the two query heads of a GQA pair (same rows), or two consecutive row blocks
// of one head.  Each K/V tile is therefore loaded once for 256 query rows.
//   warp 0      TMA producer: Q tiles once, then K_j, V_j through a stage ring
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warps 4-7   softmax + epilogue of query tile 0 (one TMEM lane = one row)
//   warps 8-11  softmax + epilogue of query tile 1
// TMEM (512 columns allocated): S0 [0,BN) S1 [BN,2BN) O0 [2BN,2BN+D) O1 [2BN+D,2BN+2D),
// with BN keys per tile (64 at head_dim 128, 128 at 64).
// The MMAs are issued in the order S(0,0) S(0,1) | PV(j,0) S(j+1,0) PV(j,1)
// S(j+1,1) | ..., so while one softmax group works on its S tile the tensor
// core runs the other tile's products.  The O rescale is lazy: the reference
// maximum only moves when a row's maximum grows by more than 2^8.
//
// Varlen scheduling is derived on the device from cu_seqlens (no host
// metadata, no host synchronisation), unlike varlen_flash_attention.py:102-144.
#include <cuda.h>

#include <cstdio>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "fmha.cuh"
#include "tcgen05.cuh"
#include "tma_host.cuh"

namespace aicas {

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

namespace {

constexpr int kBM = 128;  // query rows per tile (MMA M)
// warpgroup 0: producer, MMA (2 warps idle); one softmax warpgroup per query tile
template <int KT>
__host__ __device__ constexpr int threads_for() { return 128 + 128 * KT; }

struct FmhaArgs {
  CUtensorMap tm_q, tm_k, tm_v;  // 4-D, box {64 elements, 128 (Q) or BN (K, V) rows, 1 head, 1 batch}
  void* out;
  int64_t o_sb, o_sh, o_ss;
  int q_rows_first, k_rows_first, v_rows_first;  // 1: map dims (D, rows, heads, B); 0: (D, heads, rows, B)
  int batch, hq, hkv, seq_q, seq_kv, group;
  int pair_heads;  // 1: the two tiles are two heads of one KV group; 0: two row blocks of one head
  int num_m;       // prefill: row blocks (of 128 rows if pair_heads else 256)
  int num_units;   // prefill: CTAs per row block
  float scale_log2;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int num_seqs;
  const int32_t* kv_starts;  // causal prefill: optional first valid key per batch row (left padding)
  unsigned int* err;
};

// 128 keys per KV tile.  One tcgen05.mma (M=128, K=16) costs a fixed issue
// time that a product with N <= 128 does not cover, so tiles are as wide as the
// 512 tensor-memory columns allow: at head_dim 128, S0 S1 O0 O1 take all 512
// columns and P goes through shared memory (an SS P.V product); at head_dim 64
// P fits in tensor memory next to S and O (a TS P.V product: A from tensor
// memory), which also frees the shared memory the P tiles would take.
//   S_t at t*128 (fp32);  head_dim 128: O_t at 256 + t*128;
//   head_dim 64: P_t at 256 + t*64 (16-bit pairs), O_t at 384 + t*64.
template <int D, int KT>
struct Layout {
  static constexpr int kBN = 128;
  static constexpr bool kPTmem = D == 64;
  static constexpr uint32_t kQTile = kBM * D * 2;
  static constexpr uint32_t kKVTile = kBN * D * 2;
  static constexpr uint32_t kPTile = kPTmem ? 0 : kBM * kBN * 2;
  static constexpr uint32_t kColP = KT * kBN;
  static constexpr uint32_t kColO = kPTmem ? KT * (kBN + kBN / 2) : KT * kBN;
  // two tiles take all 512 columns; one tile 256, so two CTAs can share an SM
  static constexpr uint32_t kTmemCols = KT == 2 ? 512 : 256;
  static_assert(kColO + KT * D <= kTmemCols, "tensor memory budget");
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kP = kQ + KT * kQTile;
  static constexpr uint32_t kKV = kP + KT * kPTile;
  static constexpr int kStages = kPTmem ? (KT == 2 ? 10 : 5) : 3;
  static constexpr uint32_t kBar = kKV + kStages * kKVTile;
  static constexpr int kNumBars = 1 + 2 * kStages + 8 + 1;
  static constexpr uint32_t kMisc = kBar + kNumBars * 8;  // [tmem base][abort][schedule x 8]
  static constexpr uint32_t kBytes = kMisc + 64 + 1024;   // + slack to align the base to 1024
  static_assert(kBytes <= (KT == 2 ? 232448 : 232448 / 2 - 1024), "shared memory budget");
};

// Position in the K/V load sequence K0, K1, V0, K2, V1, ..., V(n-1): keys run
// one tile ahead of values, so each ring stage is refilled by the tile whose
// previous occupant is released earliest (a K tile is free after both S
// products of its iteration, a V tile only after both P.V products).
__host__ __device__ __forceinline__ int kv_load_index_k(int m) { return m == 0 ? 0 : 2 * m - 1; }
__host__ __device__ __forceinline__ int kv_load_index_v(int j, int n) { return min(2 * j + 2, 2 * n - 1); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions: two lanes of work per issue)
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unf2(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair on the FMA pipe, to take part of the exponentials off the
// MUFU unit (which alone would bound the softmax).  x = n + f with n the
// nearest integer (added to the exponent field) and f in [-1/2, 1/2]; 2^f by
// a cubic fitted here for minimal relative error (max 8.4e-5, far below the
// bf16/fp16 rounding P gets next).  x is clamped at -125 so the exponent stays
// normal; callers use it only on tiles without masked (-inf) entries.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: x + kRound rounds x to an integer in the mantissa
  constexpr float kC0 = 9.999196109e-01f, kC1 = 6.932621430e-01f, kC2 = 2.427139391e-01f, kC3 = 5.521300572e-02f;
  float x0, x1;
  unf2(x2, x0, x1);
  const uint64_t x = f2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = fadd2(x, f2(kRound, kRound));
  const uint64_t n = fadd2(t, f2(-kRound, -kRound));
  const uint64_t fr = ffma2(n, f2(-1.f, -1.f), x);
  uint64_t q = ffma2(f2(kC3, kC3), fr, f2(kC2, kC2));
  q = ffma2(q, fr, f2(kC1, kC1));
  q = ffma2(q, fr, f2(kC0, kC0));
  float q0, q1, t0, t1;
  unf2(q, q0, q1);
  unf2(t, t0, t1);
  // the low mantissa bits of t hold n; shifted to the exponent field they add n
  return f2(__int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23)),
            __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23)));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

__device__ __forceinline__ void tma_tile(uint32_t dst, const CUtensorMap* map, int rows_first, int d0, int row,
                                         int head, int b, uint32_t bar) {
  if (rows_first) tma_load_4d(dst, map, d0, row, head, b, bar);
  else tma_load_4d(dst, map, d0, head, row, b, bar);
}

// Every lane waits; the warp proceeds only if all lanes saw the phase.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort, unsigned int* err) {
  const bool ok = mbar_wait(bar, parity, abort, err);
  return __all_sync(0xffffffffu, ok);
}

template <typename T, int D, bool CAUSAL, bool VARLEN, int KT>
__global__ void __launch_bounds__(threads_for<KT>(), 3 - KT) fmha_fwd_kernel(const __grid_constant__ FmhaArgs a) {
  using Lay = Layout<D, KT>;
  constexpr int kThreads = threads_for<KT>();
  static_assert(KT == 2 || VARLEN, "one query tile per CTA is the varlen (ViT) form");
  // register split between warpgroup 0 (producer, MMA) and the softmax
  // warpgroups: the launch allocation is 65536 / (threads x CTAs per SM)
  // registers a thread, kept in total
  constexpr uint32_t kRegsLow = KT == 2 ? 104 : 56;
  constexpr uint32_t kRegsHigh = KT == 2 ? 200 : 200;
  static_assert(KT == 2 ? 128 * kRegsLow + 256 * kRegsHigh <= 384 * 168 : kRegsLow + kRegsHigh <= 2 * 128,
                "register split");
  constexpr int NS = Lay::kStages;
  constexpr int kBN = Lay::kBN;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  // pairs out of every 8 (16 columns) whose exponential runs on the FMA pipe
  // (measured: 2 at head_dim 128; none at 64, where the FMA pipe is busier
  // with the softmax's other work than the MUFU unit is with ex2)
  constexpr int kPolyPairs = D == 128 ? 2 : 0;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (sb - raw);
  const uint32_t bar0 = sb + Lay::kBar;
  const uint32_t q_full = bar0;
  auto kv_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + NS + s); };
  auto s_full = [&](int t) { return bar0 + 8u * (1 + 2 * NS + t); };
  auto p_full = [&](int t) { return bar0 + 8u * (3 + 2 * NS + t); };
  auto o_full = [&](int t) { return bar0 + 8u * (5 + 2 * NS + t); };
  auto s_free = [&](int t) { return bar0 + 8u * (7 + 2 * NS + t); };
  const uint32_t mma_done = bar0 + 8u * (9 + 2 * NS);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gb + Lay::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gb + Lay::kMisc + 4);
  volatile int* sched = reinterpret_cast<volatile int*>(gb + Lay::kMisc + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---------------------------------------------------------------- work unit
  int b = 0, head0, head1, kvh, row0, row1, q_base = 0, k_base = 0, q_len, kv_len;
  int kv_start = 0;  // keys before it are padding (masked), causal prefill only
  if constexpr (!VARLEN) {
    const int L = blockIdx.x;
    const int mb = a.num_m - 1 - L / a.num_units;  // longest causal rows first
    const int u = L % a.num_units;
    if (a.pair_heads) {
      const int gp_per = a.group / 2;
      const int per_b = a.hkv * gp_per;
      b = u / per_b;
      const int rem = u % per_b;
      kvh = rem / gp_per;
      head0 = kvh * a.group + 2 * (rem % gp_per);
      head1 = head0 + 1;
      row0 = row1 = mb * kBM;
    } else {
      b = u / a.hq;
      head0 = head1 = u % a.hq;
      kvh = head0 / a.group;
      row0 = mb * 2 * kBM;
      row1 = row0 + kBM;
    }
    q_len = kv_len = a.seq_q;
    if (a.kv_starts != nullptr) kv_start = min(max(__ldg(a.kv_starts + b), 0), kv_len);
  } else {
    if (warp == 0) {
      // find (sequence, row block of KT x 128 rows) of this CTA: prefix sums
      // of ceil(len_q / (KT x 128)) over the sequences, 32 sequences per step
      const int H = a.hq;
      int target = blockIdx.x / H;
      int found = -1, pr = 0, qs = 0, ql = 0, ks = 0, kl = 0;
      if (a.num_seqs <= 32) {
        // up to 32 sequences (a batch of images): the longest keys first, so
        // that the CTAs handed out last are short ones and the launch ends
        // together (ties by index); a row block's work grows with the key
        // length, and CTAs are handed out in blockIdx order
        const int i = lane;
        int np = 0, qsi = 0, qei = 0, ksi = 0, kei = 0, klen = -1;
        if (i < a.num_seqs) {
          qsi = min(max(a.cu_q[i], 0), a.seq_q);
          qei = min(max(a.cu_q[i + 1], qsi), a.seq_q);
          ksi = min(max(a.cu_k[i], 0), a.seq_kv);
          kei = min(max(a.cu_k[i + 1], ksi), a.seq_kv);
          np = (qei - qsi + KT * kBM - 1) / (KT * kBM);
          klen = kei - ksi;
        }
        int excl = 0;  // row blocks of the sequences ordered before this one
        for (int j = 0; j < 32; ++j) {
          const int kj = __shfl_sync(0xffffffffu, klen, j);
          const int npj = __shfl_sync(0xffffffffu, np, j);
          if (kj > klen || (kj == klen && j < i)) excl += npj;
        }
        const unsigned ball = __ballot_sync(0xffffffffu, i < a.num_seqs && target >= excl && target < excl + np);
        if (ball) {
          const int src = __ffs(ball) - 1;
          found = src;
          pr = target - __shfl_sync(0xffffffffu, excl, src);
          qs = __shfl_sync(0xffffffffu, qsi, src);
          ql = __shfl_sync(0xffffffffu, qei - qsi, src);
          ks = __shfl_sync(0xffffffffu, ksi, src);
          kl = __shfl_sync(0xffffffffu, kei - ksi, src);
        }
      }
      for (int base = 0; a.num_seqs > 32 && base < a.num_seqs && found < 0; base += 32) {
        const int i = base + lane;
        int np = 0, qsi = 0, qei = 0, ksi = 0, kei = 0;
        if (i < a.num_seqs) {
          qsi = min(max(a.cu_q[i], 0), a.seq_q);
          qei = min(max(a.cu_q[i + 1], qsi), a.seq_q);
          ksi = min(max(a.cu_k[i], 0), a.seq_kv);
          kei = min(max(a.cu_k[i + 1], ksi), a.seq_kv);
          np = (qei - qsi + KT * kBM - 1) / (KT * kBM);
        }
        int incl = np;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += v;
        }
        const int excl = incl - np;
        const unsigned ball = __ballot_sync(0xffffffffu, i < a.num_seqs && target >= excl && target < incl);
        if (ball) {
          const int src = __ffs(ball) - 1;
          found = base + src;
          pr = target - __shfl_sync(0xffffffffu, excl, src);
          qs = __shfl_sync(0xffffffffu, qsi, src);
          ql = __shfl_sync(0xffffffffu, qei - qsi, src);
          ks = __shfl_sync(0xffffffffu, ksi, src);
          kl = __shfl_sync(0xffffffffu, kei - ksi, src);
        } else {
          target -= __shfl_sync(0xffffffffu, incl, 31);
        }
      }
      if (lane == 0) {
        sched[0] = found;
        sched[1] = pr;
        sched[2] = qs;
        sched[3] = ql;
        sched[4] = ks;
        sched[5] = kl;
      }
    }
    __syncthreads();
    if (sched[0] < 0) return;  // past the last tile (uniform)
    head0 = head1 = kvh = blockIdx.x % a.hq;
    row0 = sched[1] * KT * kBM;
    row1 = row0 + kBM;
    q_base = sched[2];
    q_len = sched[3];
    k_base = sched[4];
    kv_len = sched[5];
  }
  int kv_end = kv_len;
  if (CAUSAL) kv_end = min(kv_len, max(row0, row1) + kBM);
  // key tiles [j0, j0 + n_kv): the ones between the first valid key and the causal end
  const int j0 = kv_start / kBN;
  const int n_kv = max(0, (kv_end + kBN - 1) / kBN - j0);

  // ---------------------------------------------------------------- set-up
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int t = 0; t < KT; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(p_full(t), 128);
      mbar_init(o_full(t), 1);
      mbar_init(s_free(t), 128);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(sb + Lay::kMisc, Lay::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // the allocation starts at lane 0 and at a multiple of its size (column 0,
  // or 256 for the second of two 256-column allocations on an SM)
  if (threadIdx.x == 0 && ((tmem >> 16) != 0u || (tmem & 0xFFFFu) % Lay::kTmemCols != 0u ||
                           (tmem & 0xFFFFu) + Lay::kTmemCols > 512u)) {
    flag_device_error(a.err, AICAS_DEVERR_TMEM);
    *abort_flag = 1;
  }
  __syncthreads();
  if (warp < 4) {
    tc::regs_dec<kRegsLow>();
    if (warp == 0) {
      // ------------------------------------------------------------ TMA producer
      if (lane == 0 && !*abort_flag) {
        tma_prefetch_desc(&a.tm_q);
        tma_prefetch_desc(&a.tm_k);
        tma_prefetch_desc(&a.tm_v);
        mbar_arrive_expect_tx(q_full, KT * Lay::kQTile);
        for (int t = 0; t < KT; ++t)
          for (int bx = 0; bx < D / 64; ++bx)
            tma_tile(sb + Lay::kQ + t * Lay::kQTile + bx * (kBM * 128), &a.tm_q, a.q_rows_first, bx * 64,
                     q_base + (t ? row1 : row0), t ? head1 : head0, b, q_full);
        int issued = 0;
        for (int idx = 0; idx < 2 * n_kv; ++idx) {
          // idx -> tile: 0 is K0, then K(j+1), V(j) pairs, the last V alone
          bool is_v;
          int j;
          if (idx == 0) {
            is_v = false;
            j = 0;
          } else if (idx == 2 * n_kv - 1) {
            is_v = true;
            j = n_kv - 1;
          } else {
            is_v = (idx & 1) == 0;
            j = is_v ? (idx - 2) / 2 : (idx + 1) / 2;
          }
          const int s = idx % NS, u = idx / NS;
          if (u > 0 && !mbar_wait(kv_empty(s), (u - 1) & 1, abort_flag, a.err)) break;
          mbar_arrive_expect_tx(kv_full(s), Lay::kKVTile);
          for (int bx = 0; bx < D / 64; ++bx)
            tma_tile(sb + Lay::kKV + s * Lay::kKVTile + bx * (kBN * 128), is_v ? &a.tm_v : &a.tm_k,
                     is_v ? a.v_rows_first : a.k_rows_first, bx * 64, k_base + (j0 + j) * kBN, kvh, b, kv_full(s));
          ++issued;
        }
        if (*abort_flag) {  // let our own copies land before the CTA can retire
          mbar_wait(q_full, 0, nullptr, a.err);
          for (int idx = max(0, issued - NS); idx < issued; ++idx)
            mbar_wait(kv_full(idx % NS), (idx / NS) & 1, nullptr, a.err);
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issue (one thread)
      if (lane == 0) {
        constexpr uint32_t kIdS = tc::idesc_f16(kBF16, kBM, kBN, false, false);
        constexpr uint32_t kIdPV = tc::idesc_f16(kBF16, kBM, D, false, true);
        // Descriptors are built once.  A descriptor depends on its tile's address
        // only through the 14-bit start-address field (address >> 4, below 2^14
        // for every shared-memory address here), so moving to another tile or
        // k-step is one 64-bit add of a constant: the issuing thread spends its
        // time issuing products, not rebuilding descriptors.
        const uint64_t dq0 = tc::smem_desc_sw128(sb + Lay::kQ, 16, 1024);
        const uint64_t dk0 = tc::smem_desc_sw128(sb + Lay::kKV, 16, 1024);
        const uint64_t dv0 = tc::smem_desc_sw128(sb + Lay::kKV, kBN * 128, 1024);
        auto issue_s = [&](int stage, int t) {
          const uint64_t qa = dq0 + ((uint64_t)(t * Lay::kQTile) >> 4);
          const uint64_t kb = dk0 + ((uint64_t)(stage * Lay::kKVTile) >> 4);
          const uint32_t dst = tmem + t * kBN;
  #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            tc::mma_f16_ss(dst, qa + (uint64_t)(((kk >> 2) * (kBM * 128) + (kk & 3) * 32) >> 4),
                           kb + (uint64_t)(((kk >> 2) * (kBN * 128) + (kk & 3) * 32) >> 4), kIdS, kk > 0 ? 1u : 0u);
        };
        const uint64_t dp0 = tc::smem_desc_sw128(sb + Lay::kP, 16, 1024);
        auto issue_pv = [&](int j, int stage, int t) {
          const uint64_t vb = dv0 + ((uint64_t)(stage * Lay::kKVTile) >> 4);
          const uint32_t dst = tmem + Lay::kColO + t * D;
          if constexpr (Lay::kPTmem) {
            const uint32_t pa = tmem + Lay::kColP + t * (kBN / 2);
  #pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk)
              tc::mma_f16_ts(dst, pa + kk * 8, vb + (uint64_t)((kk * (16 * 128)) >> 4), kIdPV,
                             (j > 0 || kk > 0) ? 1u : 0u);
          } else {
            const uint64_t pa = dp0 + ((uint64_t)(t * Lay::kPTile) >> 4);
  #pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk)
              tc::mma_f16_ss(dst, pa + (uint64_t)(((kk >> 2) * (kBM * 128) + (kk & 3) * 32) >> 4),
                             vb + (uint64_t)((kk * (16 * 128)) >> 4), kIdPV, (j > 0 || kk > 0) ? 1u : 0u);
          }
        };
        bool ok = !*abort_flag && mbar_wait(q_full, 0, abort_flag, a.err);
        if (ok && n_kv > 0) {
          ok = mbar_wait(kv_full(0), 0, abort_flag, a.err);
          if constexpr (KT == 2) {
            if (ok) {
              tc::fence_after_sync();
              issue_s(0, 0);
              tc::commit(s_full(0));
              issue_s(0, 1);
              tc::commit(s_full(1));
              tc::commit(kv_empty(0));
            }
            for (int j = 0; ok && j < n_kv; ++j) {
              const int iv = kv_load_index_v(j, n_kv), ik = kv_load_index_k(j + 1);
              const int sv = iv % NS, sk = ik % NS;
              const bool more = j + 1 < n_kv;
              // Per-tile order, as the softmax groups release their inputs:
              // S(j+1,0) as soon as group 0 has READ S(j,0) (not after its softmax),
              // PV(j,0) once P(j,0) is written, then the same for tile 1.
              if (more) {
                ok = mbar_wait(kv_full(sk), (ik / NS) & 1, abort_flag, a.err) &&
                     mbar_wait(s_free(0), j & 1, abort_flag, a.err);
                if (!ok) break;
                tc::fence_after_sync();
                issue_s(sk, 0);
                tc::commit(s_full(0));
              }
              ok = mbar_wait(kv_full(sv), (iv / NS) & 1, abort_flag, a.err) &&
                   mbar_wait(p_full(0), j & 1, abort_flag, a.err);
              if (!ok) break;
              tc::fence_after_sync();
              issue_pv(j, sv, 0);
              tc::commit(o_full(0));
              if (more) {
                ok = mbar_wait(s_free(1), j & 1, abort_flag, a.err);
                if (!ok) break;
                tc::fence_after_sync();
                issue_s(sk, 1);
                tc::commit(s_full(1));
                tc::commit(kv_empty(sk));
              }
              ok = mbar_wait(p_full(1), j & 1, abort_flag, a.err);
              if (!ok) break;
              tc::fence_after_sync();
              issue_pv(j, sv, 1);
              tc::commit(o_full(1));
              tc::commit(kv_empty(sv));
            }
          } else {
            // one tile: S(j+1) as soon as the softmax has read S(j), PV(j) once P(j) is written
            if (ok) {
              tc::fence_after_sync();
              issue_s(0, 0);
              tc::commit(s_full(0));
              tc::commit(kv_empty(0));
            }
            for (int j = 0; ok && j < n_kv; ++j) {
              const int iv = kv_load_index_v(j, n_kv), ik = kv_load_index_k(j + 1);
              const int sv = iv % NS, sk = ik % NS;
              if (j + 1 < n_kv) {
                ok = mbar_wait(kv_full(sk), (ik / NS) & 1, abort_flag, a.err) &&
                     mbar_wait(s_free(0), j & 1, abort_flag, a.err);
                if (!ok) break;
                tc::fence_after_sync();
                issue_s(sk, 0);
                tc::commit(s_full(0));
                tc::commit(kv_empty(sk));
              }
              ok = mbar_wait(kv_full(sv), (iv / NS) & 1, abort_flag, a.err) &&
                   mbar_wait(p_full(0), j & 1, abort_flag, a.err);
              if (!ok) break;
              tc::fence_after_sync();
              issue_pv(j, sv, 0);
              tc::commit(o_full(0));
              tc::commit(kv_empty(sv));
            }
          }
        }
        // all products issued so far have completed before the CTA tears down
        tc::commit(mma_done);
        mbar_wait(mma_done, 0, nullptr, a.err);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    // warpgroup 1 owns query tile 0, warpgroup 2 tile 1; a warp may only touch
    // the TMEM lanes of its rank within its warpgroup (warp % 4), which is the
    // quarter of the tile's rows it owns
    tc::regs_inc<kRegsHigh>();
    const int t = (warp - 4) >> 2;
    const int qw = warp & 3;
    const int r = qw * 32 + lane;
    const int tile_row0 = t ? row1 : row0;
    const int row = tile_row0 + r;
    const bool row_valid = row < q_len;
    const uint32_t tl = tmem + ((uint32_t)(qw * 32) << 16);
    const uint32_t col_s = t * kBN, col_p = Lay::kColP + t * (kBN / 2), col_o = Lay::kColO + t * D;
    uint8_t* prow = gb + Lay::kP + t * Lay::kPTile + (r >> 3) * 1024 + (r & 7) * 128;  // P row (head_dim 128)
    const float c = a.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = !*abort_flag;
    uint32_t v[kBN];  // the S row of this thread, then reused for O chunks
    const uint32_t masked_bits = __float_as_uint(c >= 0.f ? -INFINITY : INFINITY);  // s*c -> -inf
    for (int j = 0; ok && j < n_kv; ++j) {
      if (!warp_wait(s_full(t), j & 1, abort_flag, a.err)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
#pragma unroll
      for (int cc = 0; cc < kBN / 32; ++cc) tc::tmem_ld32(tl + col_s + 32 * cc, v + 32 * cc);
      tc::tmem_wait_ld();
      // S(j) is in registers: the tensor core may overwrite it with S(j+1) now
      tc::fence_before_sync();
      mbar_arrive(s_free(t));
      const int kv0 = (j0 + j) * kBN;
      const bool mask = (kv0 + kBN > kv_len) || (CAUSAL && kv0 + kBN - 1 > tile_row0) || kv0 < kv_start;
      if (mask) {
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          const int col = kv0 + i;
          if (col >= kv_len || (CAUSAL && col > row) || col < kv_start) v[i] = masked_bits;
        }
      }
      // row maximum of s*c: 4 independent chains of 3-input max
      float mx;
      {
        float m4[4];
        if (c >= 0.f) {
#pragma unroll
          for (int k = 0; k < 4; ++k) m4[k] = -INFINITY;
#pragma unroll
          for (int i = 0; i < kBN; i += 2)
            m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
          mx = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) m4[k] = INFINITY;
#pragma unroll
          for (int i = 0; i < kBN; i += 2)
            m4[(i >> 1) & 3] = fmin3(m4[(i >> 1) & 3], __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
          mx = fmin3(m4[0], m4[1], fminf(m4[2], m4[3]));
        }
        mx = (mx == -INFINITY || mx == INFINITY) ? -INFINITY : mx * c;
      }
      bool rescale = false;
      float alpha = 1.f;
      if (mx > m_ref + 8.f) {  // first finite maximum, or growth beyond 2^8: move the reference
        alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - mx);
        rescale = j > 0 && m_ref != -INFINITY;
        l *= alpha;
        m_ref = mx;
      }
      const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
      // P = 2^(s*c - m) for the whole row, packed to 16-bit pairs in registers
      // (the S registers are consumed as P fills): none of it waits for the
      // previous P.V product, which still reads this tile's P buffer.  Pairs
      // are scaled with one f32x2 FMA; on tiles without masked entries
      // kPolyPairs of every 8 pairs take the polynomial exponential, the rest
      // ex2.approx; partial sums in f32x2 accumulators.
      uint64_t rs2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
      const uint64_t c2 = f2(c, c), nm2 = f2(-m_use, -m_use);
      // the packed pair e overwrites v[e]: v[2e] and v[2e + 1] are read first,
      // and no later pair reads below index 2e + 2, so P takes no registers of its own
      uint32_t* pk = v;
      if (mask) {
#pragma unroll
        for (int e = 0; e < kBN / 2; ++e) {
          float x0, x1;
          unf2(ffma2(f2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), c2, nm2), x0, x1);
          const float p0 = ex2(x0), p1 = ex2(x1);
          rs2[e & 1] = fadd2(rs2[e & 1], f2(p0, p1));
          pk[e] = pack2<T>(p0, p1);
        }
      } else {
#pragma unroll
        for (int e = 0; e < kBN / 2; ++e) {
          const uint64_t x2 = ffma2(f2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), c2, nm2);
          float p0, p1;
          if ((e & 7) < kPolyPairs) {
            unf2(exp2_poly2(x2), p0, p1);
          } else {
            float x0, x1;
            unf2(x2, x0, x1);
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          rs2[e & 1] = fadd2(rs2[e & 1], f2(p0, p1));
          pk[e] = pack2<T>(p0, p1);
        }
      }
      // the P buffer and O are free once PV(j-1) of this tile has completed
      if (j > 0) {
        if (!warp_wait(o_full(t), (j - 1) & 1, abort_flag, a.err)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
      }
#pragma unroll
      for (int h = 0; h < kBN / 64; ++h) {
        if constexpr (Lay::kPTmem) {
          tc::tmem_st32(tl + col_p + 32 * h, pk + 32 * h);
        } else {
          // K-major 128B-swizzled P tile: 16-byte chunk c of row r at c ^ (r % 8)
          uint8_t* sub = prow + h * (kBM * 128);
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(sub + ((ch ^ (r & 7)) << 4)) =
                make_uint4(pk[32 * h + 4 * ch], pk[32 * h + 4 * ch + 1], pk[32 * h + 4 * ch + 2],
                           pk[32 * h + 4 * ch + 3]);
        }
      }
      float rs4[4];
      unf2(rs2[0], rs4[0], rs4[1]);
      unf2(rs2[1], rs4[2], rs4[3]);
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      // the S registers are dead now: rescale O (rare, lazy) with the same registers
      if (__any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? alpha : 1.f;
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          tc::tmem_ld32(tl + col_o + 32 * cc, v);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
          tc::tmem_st32(tl + col_o + 32 * cc, v);
        }
        tc::tmem_wait_st();
      }
      if constexpr (Lay::kPTmem) tc::tmem_wait_st();  // P is in tensor memory before PV(j) may read it
      else fence_proxy_async_smem();                   // P in shared memory is visible to the tensor core
      tc::fence_before_sync();
      mbar_arrive(p_full(t));
    }
    // epilogue: O / l -> global
    T* orow = static_cast<T*>(a.out) + (int64_t)b * a.o_sb + (int64_t)(t ? head1 : head0) * a.o_sh +
              (int64_t)(q_base + row) * a.o_ss;
    if (ok && n_kv > 0) {
      if (warp_wait(o_full(t), (n_kv - 1) & 1, abort_flag, a.err)) {
        tc::fence_after_sync();
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) tc::tmem_ld32(tl + col_o + 32 * cc, v + 32 * cc);
        tc::tmem_wait_ld();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        // O / l through this warp's 32 rows of the tile's Q buffer (free: every
        // S product of this tile has completed), 16-byte chunks XOR-swizzled by
        // row; then each store instruction writes whole rows (kChunks lanes per
        // row), not one 16-byte piece of 32 different rows
        constexpr int kChunks = D * 2 / 16;
        constexpr int kRowsPerStore = 32 / kChunks;
        uint8_t* stage = gb + Lay::kQ + t * Lay::kQTile + qw * (32 * D * 2);
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = pack2<T>(__uint_as_float(v[8 * ch + 2 * i]) * inv, __uint_as_float(v[8 * ch + 2 * i + 1]) * inv);
          *reinterpret_cast<uint4*>(stage + lane * (D * 2) + ((ch ^ (lane & (kChunks - 1))) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
        __syncwarp();
        const int wrow0 = tile_row0 + qw * 32;  // first row of this warp
        T* obase = static_cast<T*>(a.out) + (int64_t)b * a.o_sb + (int64_t)(t ? head1 : head0) * a.o_sh;
#pragma unroll
        for (int k = 0; k < kChunks; ++k) {
          const int rr = k * kRowsPerStore + lane / kChunks;
          const int ch = lane % kChunks;
          const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * (D * 2) + ((ch ^ (rr & (kChunks - 1))) << 4));
          if (wrow0 + rr < q_len)
            *reinterpret_cast<uint4*>(obase + (int64_t)(q_base + wrow0 + rr) * a.o_ss + ch * 8) = val;
        }
      }
    } else if (ok && row_valid) {
      uint4* dst = reinterpret_cast<uint4*>(orow);
      for (int q4 = 0; q4 < D / 8; ++q4) dst[q4] = make_uint4(0u, 0u, 0u, 0u);  // empty key range
    }
  }

  // ---------------------------------------------------------------- teardown
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, Lay::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side

// 4-D map over [B, heads, rows, D] (element strides), the two middle dimensions
// ordered by increasing stride as the tensor-map encoder expects.
bool make_map(CUtensorMap* m, const void* ptr, bool bf16, int d, int rows, int heads, int batch, int64_t s_b,
              int64_t s_h, int64_t s_s, int box_rows, int* rows_first, char* err, size_t errlen) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (enc == nullptr) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  // size-1 dimensions may carry any stride in a torch view: give them a valid one
  const int64_t big = (int64_t)rows * s_s + (int64_t)heads * s_h + 8;
  if (heads == 1) s_h = ((s_s * (int64_t)rows + 7) / 8) * 8;
  if (rows == 1) s_s = ((s_h * (int64_t)heads + 7) / 8) * 8;
  if (batch == 1) s_b = ((big + 7) / 8) * 8;
  const bool rf = s_s <= s_h;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], estr[4] = {1, 1, 1, 1};
  dims[0] = (cuuint64_t)d;
  box[0] = 64;
  if (rf) {
    dims[1] = rows; dims[2] = heads; strides[0] = s_s * 2; strides[1] = s_h * 2; box[1] = box_rows; box[2] = 1;
  } else {
    dims[1] = heads; dims[2] = rows; strides[0] = s_h * 2; strides[1] = s_s * 2; box[1] = 1; box[2] = box_rows;
  }
  dims[3] = batch;
  strides[2] = s_b * 2;
  box[3] = 1;
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (%d) for dims [%d,%d,%d,%d] strides [%lld,%lld,%lld]",
             (int)r, d, rows, heads, batch, (long long)s_s, (long long)s_h, (long long)s_b);
    return false;
  }
  *rows_first = rf ? 1 : 0;
  return true;
}

template <typename T, int D, bool CAUSAL, bool VARLEN, int KT>
cudaError_t launch_t(const FmhaArgs& a, int grid, cudaStream_t st) {
  auto kern = fmha_fwd_kernel<T, D, CAUSAL, VARLEN, KT>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<D, KT>::kBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  kern<<<grid, threads_for<KT>(), Layout<D, KT>::kBytes, st>>>(a);
  return cudaGetLastError();
}

// Query tiles per CTA of the varlen kernel at head_dim 64 (the ViT): one, so
// that two CTAs share an SM and each hides the other's fill and drain.
#ifndef AICAS_VARLEN64_TILES
#define AICAS_VARLEN64_TILES 1
#endif
constexpr int kVarlen64Tiles = AICAS_VARLEN64_TILES;

int tiles_per_cta(int d, bool varlen) { return (varlen && d == 64) ? kVarlen64Tiles : 2; }

template <typename T>
cudaError_t dispatch(int d, bool varlen, const FmhaArgs& a, int grid, cudaStream_t st) {
  if (d == 128)
    return varlen ? launch_t<T, 128, false, true, 2>(a, grid, st) : launch_t<T, 128, true, false, 2>(a, grid, st);
  return varlen ? launch_t<T, 64, false, true, kVarlen64Tiles>(a, grid, st) : launch_t<T, 64, true, false, 2>(a, grid, st);
}

}  // namespace

uint32_t fmha_capabilities() { return AICAS_CAP_PREFILL_TCGEN05 | AICAS_CAP_VARLEN_TCGEN05; }

int run_fmha(const aicas_fmha_params* p, bool varlen, cudaStream_t stream, unsigned int* dev_err, char* err,
             size_t errlen) {
  if (p->seq_len_q == 0) return AICAS_OK;
  const bool bf16 = p->dtype == AICAS_DTYPE_BF16;
  FmhaArgs a;
  memset(&a, 0, sizeof(a));
  const int kv_box = Layout<128, 2>::kBN;
  if (!make_map(&a.tm_q, p->q, bf16, p->head_dim, p->seq_len_q, p->num_q_heads, p->batch, p->q_stride_b,
                p->q_stride_h, p->q_stride_s, kBM, &a.q_rows_first, err, errlen) ||
      !make_map(&a.tm_k, p->k, bf16, p->head_dim, p->seq_len_kv, p->num_kv_heads, p->batch, p->k_stride_b,
                p->k_stride_h, p->k_stride_s, kv_box, &a.k_rows_first, err, errlen) ||
      !make_map(&a.tm_v, p->v, bf16, p->head_dim, p->seq_len_kv, p->num_kv_heads, p->batch, p->v_stride_b,
                p->v_stride_h, p->v_stride_s, kv_box, &a.v_rows_first, err, errlen))
    return AICAS_ERR_UNSUPPORTED;
  a.out = p->out;
  a.o_sb = p->o_stride_b;
  a.o_sh = p->o_stride_h;
  a.o_ss = p->o_stride_s;
  a.batch = p->batch;
  a.hq = p->num_q_heads;
  a.hkv = p->num_kv_heads;
  a.seq_q = p->seq_len_q;
  a.seq_kv = p->seq_len_kv;
  a.group = p->num_q_heads / p->num_kv_heads;
  a.scale_log2 = p->sm_scale * 1.4426950408889634f;
  a.kv_starts = varlen ? nullptr : p->kv_starts;
  a.err = dev_err;
  long long grid;
  if (varlen) {
    a.cu_q = p->cu_seqlens_q;
    a.cu_k = p->cu_seqlens_k;
    a.num_seqs = p->num_seqs;
    if (p->num_seqs == 0) return AICAS_OK;
    const int rows = tiles_per_cta(p->head_dim, true) * kBM;
    grid = ((long long)(p->seq_len_q + rows - 1) / rows + p->num_seqs) * p->num_q_heads;
  } else {
    a.pair_heads = (a.group % 2 == 0) ? 1 : 0;
    a.num_m = a.pair_heads ? (p->seq_len_q + kBM - 1) / kBM : (p->seq_len_q + 2 * kBM - 1) / (2 * kBM);
    a.num_units = a.pair_heads ? p->batch * p->num_kv_heads * (a.group / 2) : p->batch * p->num_q_heads;
    grid = (long long)a.num_m * a.num_units;
  }
  if (grid > 0x7fffffffLL) {
    snprintf(err, errlen, "attention grid too large");
    return AICAS_ERR_UNSUPPORTED;
  }
  if (grid == 0) return AICAS_OK;
  const cudaError_t e = bf16 ? dispatch<__nv_bfloat16>(p->head_dim, varlen, a, (int)grid, stream)
                             : dispatch<__half>(p->head_dim, varlen, a, (int)grid, stream);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "attention launch: %s (%s)", cudaGetErrorString(e), cudaGetErrorName(e));
    return AICAS_ERR_CUDA;
  }
  return AICAS_OK;
}

}  // namespace aicas
