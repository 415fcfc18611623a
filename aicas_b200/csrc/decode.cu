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
//   * work items are (request, KV head, split of the cache), run by persistent
//     CTAs (see decode_gqa_kernel); the whole GQA group of query heads is served
//     from ONE copy of each K/V tile (the reference streams the KV head once per
//     query head);
//   * a producer warp streams 16 KB K and V tiles with cp.async.bulk (TMA into
//     this CTA's shared memory, L2 evict-first) into a 3-stage mbarrier ring;
//   * 8 consumer warps (4 for groups of 4 or more query heads) each own a
//     slice of every tile: 16-byte vector reads
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
  // consumer warps: the per-tile work of a warp is a chain of dependent
  // shuffles and exponentials, so more warps hide more of its latency; with 4
  // or more query heads per KV head the per-warp reduction buffer of 8 warps
  // would leave room for only one CTA per SM
  static constexpr int kWarps = G <= 2 ? 8 : 4;
  static constexpr int kThreads = (kWarps + 1) * 32;  // + 1 producer warp
  static constexpr int kTileBytes = 16384;
  static constexpr int kTile = kTileBytes / kRowBytes;  // tokens per stage
  static constexpr int kTPW = kTile / kWarps;           // tokens per warp per tile
  static constexpr int kNP = kTPW / kTPP;               // passes per tile
  static constexpr int kNV = kNP * G;                   // partial scores per lane
  static constexpr int kLogLPT = kLPT == 1 ? 0 : kLPT == 2 ? 1 : kLPT == 4 ? 2 : kLPT == 8 ? 3 : kLPT == 16 ? 4 : 5;
  static constexpr int kLogNP = kNP == 4 ? 2 : kNP == 8 ? 3 : -1;
  // halving steps of the reduce-scatter: stop once a lane holds one full pass (G values)
  static constexpr int kHalve = kLogLPT < kLogNP ? kLogLPT : kLogNP;
  static constexpr int kRV = kNV >> kHalve;            // values kept per lane (multiple of G)
  static constexpr int kDup = kLPT >> kHalve;          // lanes holding identical values
  static constexpr int kStages = 3;
  static constexpr int kQueue = 4;                     // work items announced ahead by the producer
  static constexpr int kQBytes = G * D * (int)sizeof(T);  // query rows of one item (in the queue entry)
  static constexpr int kEntryBytes = 64 + kQBytes;     // [metadata][q rows]
  static constexpr int kRedFloats = kWarps * G * (D + 2);
  static constexpr int kPFloats = kTile * G;
  // smem: K ring | V ring | item queue | barriers | reductions | probabilities
  static constexpr int kOffQueue = 2 * kStages * kTileBytes;
  static constexpr int kOffBars = kOffQueue + kQueue * kEntryBytes;
  static constexpr int kNumBars = 2 * kStages + 2 * kQueue;
  static constexpr int kOffRed = kOffBars + kNumBars * 8;
  static constexpr int kSmemBytes = kOffRed + (kRedFloats + kPFloats) * 4 + 16;
  static_assert(kEPV * kLPT == D, "head_dim must be a multiple of the vector width");
  static_assert(kLPT <= 32 && kTPP * kLPT == 32, "lanes per token must divide 32");
  static_assert(kLogNP >= 0, "tile geometry");
  static_assert(kRV % G == 0, "each lane must keep whole passes");
  static_assert(kQBytes % 16 == 0 && kEntryBytes % 16 == 0, "queue entries hold 16-byte aligned copies");
};

// One work item: a split of one (request, KV head) cache.  ntok < 0 ends the stream.
struct DecodeItem {
  int b, kvh, split, t0, ntok, nsplit;
};

// Consumer-warp barrier (named barrier 1, the consumer warps only): every
// consumer warp reaches each use exactly once per item, also on the abort
// path, so the producer warp never takes part and never blocks it.
template <int kWarps>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory");
}
// Same barrier, returning the OR of every consumer thread's predicate, so that
// all consumer warps take the same branch after it.
template <int kWarps>
__device__ __forceinline__ bool consumer_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kWarps * 32)
      : "memory");
  return r != 0;
}

// Merges the split partials of one (request, KV head) pair into its output and
// resets the pair's split counter for the next call; run by the consumer
// threads of the CTA whose increment of that counter came last.  Up to eight
// splits' partials are loaded before any is used (one L2 round trip).
// Where a (request, KV head) pair's result goes: the output (and/or the fp32
// partial + LSE) of this device, or, with the cross-GPU merge fused in (XCHG),
// this rank's slot in every rank's exchange buffer (the finalize phase of each
// rank merges the ranks' results).
template <typename T, int D, bool XCHG>
__device__ __forceinline__ void pair_result(const DecodeArgs& a, int b, int qh, int d, float ov, float lse, int par) {
  if constexpr (XCHG) {
    const int64_t bh = (int64_t)b * a.hq + qh;
    const int64_t n_o = (int64_t)a.batch * a.hq * D;
    for (int r = 0; r < a.xworld; ++r) {
      float* slot = reinterpret_cast<float*>(static_cast<uint8_t*>(a.xpeers[r]) + a.xslot_off) +
                    ((int64_t)par * a.xworld + a.xrank) * a.xslot_floats;
      slot[bh * D + d] = ov;
      if (d == 0) slot[n_o + bh] = lse;
    }
  } else {
    if (a.out != nullptr)
      static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)qh * a.o_sh + d] = Elem<T>::from_float(ov);
    if (a.partial_o != nullptr) a.partial_o[((int64_t)b * a.hq + qh) * D + d] = ov;
    if (a.lse != nullptr && d == 0) a.lse[(int64_t)b * a.hq + qh] = lse;
  }
}

template <typename T, int D, int G, int kThreads, bool XCHG>
__device__ void merge_splits(const DecodeArgs& a, int b, int kvh, int nsplit, int par) {
  constexpr int kMC = 8;
  const int bh = b * a.hkv + kvh;
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int sp0 = 0; sp0 < nsplit; sp0 += kMC) {
      float ls[kMC], os[kMC];
#pragma unroll
      for (int j = 0; j < kMC; ++j) {
        ls[j] = -INFINITY;
        os[j] = 0.f;
        if (sp0 + j < nsplit) {
          const int64_t base = ((int64_t)bh * a.max_splits + sp0 + j) * G + h;
          ls[j] = __ldcg(a.ws_lse + base);
          os[j] = __ldcg(a.ws_o + base * D + d);
        }
      }
      float mc = M;
#pragma unroll
      for (int j = 0; j < kMC; ++j) mc = fmaxf(mc, ls[j]);
      if (mc != -INFINITY) {
        const float r = exp2f(M - mc);  // 0 while nothing has been accumulated
        L *= r;
        O *= r;
#pragma unroll
        for (int j = 0; j < kMC; ++j) {
          const float w = exp2f(ls[j] - mc);
          L += w;
          O += w * os[j];
        }
        M = mc;
      }
    }
    const float ov = (L > 0.f) ? O / L : 0.f;
    const float lse = (L > 0.f) ? M + log2f(L) : -INFINITY;
    pair_result<T, D, XCHG>(a, b, kvh * G + h, d, ov, lse, par);
  }
  if (threadIdx.x == 0) a.ws_count[bh] = 0u;  // ready for the next call
}

// XCHG: publishes a pair's result to every rank, by one thread after this
// CTA's consumer threads have written it and passed a barrier: one
// system-scope fence (cumulative over their stores), then the flags.
__device__ __forceinline__ void publish_pair(const DecodeArgs& a, int pair, unsigned long long e) {
  fence_acq_rel_sys();
  for (int r = 0; r < a.xworld; ++r)
    st_relaxed_sys(reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(a.xpeers[r]) + kExchangePairFlags) +
                       (int64_t)pair * 8 + a.xrank,
                   e);
}

// Persistent CTAs (as many as fit on the device at once) run through the
// (request, KV head, split) work items.  With a workspace the items are handed
// out by an atomic counter (ragged cache lengths make a static split
// uneven), else round-robin.  The producer warp claims items, announces each
// one in a small shared-memory queue (metadata and the item's query rows,
// copied by TMA), and streams its K/V tiles into a ring that runs on across
// items, so the copies for the next item are in flight while the consumers
// finish the current one.
//
// XCHG (the cross-GPU merge of a sequence-sharded cache fused in): each pair's
// result goes straight into this rank's slot of every rank's exchange buffer,
// with a per-pair flag; once a CTA's own item queue is drained it claims pairs
// from a second counter, waits (bounded) until every rank has published that
// pair and merges the ranks' results into the output.  No CTA waits for
// another GPU while it holds a claimed item, so ranks cannot wait on each
// other in a cycle; the last CTA out advances the buffer's epoch.
template <typename T, int D, int G, bool XCHG>
__global__ void __launch_bounds__(DecodeCfg<T, D, G>::kThreads, G <= 2 ? 2 : 1)
    decode_gqa_kernel(const DecodeArgs a) {
  using C = DecodeCfg<T, D, G>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sk = smem;
  uint8_t* sv = smem + C::kStages * C::kTileBytes;
  uint8_t* queue = smem + C::kOffQueue;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  float* red = reinterpret_cast<float*>(smem + C::kOffRed);  // [warp][G][D+2]
  float* ps = red + C::kRedFloats;                             // [tile token][G]
  __shared__ int s_abort;
  __shared__ int s_merge[4];  // [merge?, b, kvh, nsplit] of a finished pair, published by thread 0

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + C::kStages);
  const uint32_t qfull0 = smem_u32(bars + 2 * C::kStages);
  const uint32_t qempty0 = smem_u32(bars + 2 * C::kStages + C::kQueue);
  const int total_items = a.batch * a.hkv * a.max_splits;
  const bool dynamic = a.ws_count != nullptr;
  unsigned int* next_item = dynamic ? a.ws_sched : nullptr;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, C::kWarps);
    }
    for (int i = 0; i < C::kQueue; ++i) {
      mbar_init(qfull0 + 8 * i, 1);
      mbar_init(qempty0 + 8 * i, C::kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // launched with programmatic dependent launch: set-up above overlaps the
  // kernel before this one (the query, lengths, cache and workspace come after)
  if (threadIdx.x == 0) grid_launch_dependents();
  if (a.prefetch_first && threadIdx.x == C::kWarps * 32) {
    // this CTA's first item is item blockIdx.x (see the claim loop below); its
    // split covers the same tokens whatever the lengths turn out to be, so its
    // K/V can be brought into L2 while the kernel before this one finishes
    const int bh = (int)blockIdx.x % (a.batch * a.hkv), split = (int)blockIdx.x / (a.batch * a.hkv);
    const int b = bh / a.hkv, kvh = bh % a.hkv;
    const int t0 = decode_split_start(split, a.split_tokens, a.split_floor, C::kTile);
    const int ntok = min(a.cap, t0 + decode_split_size(split, a.split_tokens, a.split_floor, C::kTile)) - t0;
    if (ntok > 0) {
      const uint8_t* gk = static_cast<const uint8_t*>(a.k) +
                          ((int64_t)b * a.k_sb + (int64_t)kvh * a.k_sh + (int64_t)t0 * D) * sizeof(T);
      const uint8_t* gv = static_cast<const uint8_t*>(a.v) +
                          ((int64_t)b * a.v_sb + (int64_t)kvh * a.v_sh + (int64_t)t0 * D) * sizeof(T);
      const uint32_t bytes = (uint32_t)ntok * C::kRowBytes;
      for (uint32_t off = 0; off < bytes; off += 65536u) {
        const uint32_t n = bytes - off < 65536u ? bytes - off : 65536u;
        bulk_prefetch_l2(gk + off, n);
        bulk_prefetch_l2(gv + off, n);
      }
    }
  }
  grid_dependency_wait();
  // XCHG: this call's epoch and slot parity (every CTA reads the epoch before
  // the last CTA out advances it)
  unsigned long long xe = 0;
  int xpar = 0;
  if constexpr (XCHG) {
    xe = *reinterpret_cast<volatile unsigned long long*>(static_cast<uint8_t*>(a.xpeers[a.xrank]) + 256) + 1;  // word 0
    xpar = (int)(xe & 1);
  }

  if (warp == C::kWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t g = 0;       // K/V tiles issued so far (ring position)
      uint32_t qi = 0;      // items announced so far (queue position)
      int k = 0;            // round-robin position (static scheduling)
      bool first_claim = true;
      bool ok = true;
      for (;;) {
        // claim the next non-empty item (or run out)
        int item = -1;
        DecodeItem it;
        for (;;) {
          int cand;
          if (dynamic) {
            // the first item is this CTA's own index; the counter hands out the rest
            cand = first_claim ? (int)blockIdx.x : (int)gridDim.x + (int)atomicAdd(next_item, 1u);
            first_claim = false;
          } else {
            cand = (int)blockIdx.x + k * (int)gridDim.x;
            ++k;
          }
          if (cand >= total_items) break;
          // split-major order: item = split * (B * Hkv) + (b * Hkv + kvh)
          const int bh = cand % (a.batch * a.hkv);
          it.split = cand / (a.batch * a.hkv);
          it.b = bh / a.hkv;
          it.kvh = bh % a.hkv;
          int len = a.cap;
          if (a.kv_lens != nullptr) len = min(max(__ldg(a.kv_lens + it.b), 0), a.cap);
          // valid slots [start, len): a left-padded request starts past its padding
          const int start = a.kv_starts != nullptr ? min(max(__ldg(a.kv_starts + it.b), 0), len) : 0;
          it.nsplit = decode_split_count(len - start, a.split_tokens, a.split_floor, C::kTile);
          if (it.split >= it.nsplit) continue;  // past this request's length
          it.t0 = start + decode_split_start(it.split, a.split_tokens, a.split_floor, C::kTile);
          // the last split runs to the end of the cache (it may have absorbed a short remainder)
          const int t1 = it.split == it.nsplit - 1
                             ? len
                             : it.t0 + decode_split_size(it.split, a.split_tokens, a.split_floor, C::kTile);
          it.ntok = max(0, t1 - it.t0);
          item = cand;
          break;
        }
        // announce it (or the end of the stream)
        const uint32_t slot = qi % C::kQueue;
        if (qi >= (uint32_t)C::kQueue && !mbar_wait(qempty0 + 8 * slot, (qi / C::kQueue - 1) & 1, &s_abort, a.err)) {
          ok = false;
          break;
        }
        DecodeItem* meta = reinterpret_cast<DecodeItem*>(queue + slot * C::kEntryBytes);
        if (item < 0) {
          meta->ntok = -1;
          mbar_arrive(qfull0 + 8 * slot);  // release: the consumers see the end marker
          ++qi;
          break;
        }
        *meta = it;
        const T* qsrc = static_cast<const T*>(a.q) + (int64_t)it.b * a.q_sb + (int64_t)(it.kvh * G) * a.q_sh;
        const uint32_t qdst = smem_u32(queue + slot * C::kEntryBytes + 64);
        mbar_arrive_expect_tx(qfull0 + 8 * slot, C::kQBytes);  // also publishes the metadata (release)
        if (a.q_sh == D) {
          bulk_g2s(qdst, qsrc, C::kQBytes, qfull0 + 8 * slot, pol);
        } else {
          for (int h = 0; h < G; ++h)
            bulk_g2s(qdst + h * C::kRowBytes, qsrc + (int64_t)h * a.q_sh, C::kRowBytes, qfull0 + 8 * slot, pol);
        }
        ++qi;
        // its K/V tiles
        const uint8_t* gk = static_cast<const uint8_t*>(a.k) +
                            ((int64_t)it.b * a.k_sb + (int64_t)it.kvh * a.k_sh + (int64_t)it.t0 * D) * sizeof(T);
        const uint8_t* gv = static_cast<const uint8_t*>(a.v) +
                            ((int64_t)it.b * a.v_sb + (int64_t)it.kvh * a.v_sh + (int64_t)it.t0 * D) * sizeof(T);
        const int ntiles = (it.ntok + C::kTile - 1) / C::kTile;
        for (int t = 0; t < ntiles; ++t, ++g) {
          const uint32_t s = g % C::kStages, u = g / C::kStages;
          if (u > 0 && !mbar_wait(empty0 + 8 * s, (u - 1) & 1, &s_abort, a.err)) {
            ok = false;
            break;
          }
          const uint32_t nb = (uint32_t)min(C::kTile, it.ntok - t * C::kTile) * C::kRowBytes;
          mbar_arrive_expect_tx(full0 + 8 * s, 2 * nb);
          bulk_g2s(smem_u32(sk + s * C::kTileBytes), gk + (int64_t)t * C::kTileBytes, nb, full0 + 8 * s, pol);
          bulk_g2s(smem_u32(sv + s * C::kTileBytes), gv + (int64_t)t * C::kTileBytes, nb, full0 + 8 * s, pol);
        }
        if (!ok) break;
      }
      if (!ok || s_abort) {
        // do not leave while our own copies may still land in shared memory
        for (uint32_t t = g > (uint32_t)C::kStages ? g - C::kStages : 0u; t < g; ++t)
          mbar_wait(full0 + 8 * (t % C::kStages), (t / C::kStages) & 1, nullptr, a.err);
        for (uint32_t i = qi > (uint32_t)C::kQueue ? qi - C::kQueue : 0u; i < qi; ++i)
          mbar_wait(qfull0 + 8 * (i % C::kQueue), (i / C::kQueue) & 1, nullptr, a.err);
        s_abort = 1;
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int c = lane % C::kLPT;    // 16-byte column of the head_dim row
    const int sub = lane / C::kLPT;  // token slot within a pass
    const int gl = c;                // lane index inside its token group
    // index of the first value this lane keeps after the reduce-scatter
    int idx_base = 0;
#pragma unroll
    for (int k = 0; k < C::kHalve; ++k)
      if (gl & (C::kLPT >> (k + 1))) idx_base += C::kNV >> (k + 1);
    const bool canonical = (gl % C::kDup) == 0;
    float* pw = ps + warp * C::kTPW * G;  // this warp's probabilities [token][G]
    uint32_t g = 0;                       // ring position
    // thread 0: the split-counter increment of the last split item, whose
    // result is read one item later so that its round trip overlaps the tiles
    unsigned int pend_prev = 0;
    int pend_b = -1, pend_kvh = 0, pend_nsplit = 0;
    const auto publish_pending = [&]() {
      s_merge[0] = (pend_b >= 0 && pend_prev == (unsigned int)(pend_nsplit - 1)) ? 1 : 0;
      s_merge[1] = pend_b;
      s_merge[2] = pend_kvh;
      s_merge[3] = pend_nsplit;
      pend_b = -1;
    };
    for (uint32_t qi = 0;; ++qi) {
      // ---- next item from the queue (every consumer warp takes every item)
      const uint32_t slot = qi % C::kQueue;
      const bool got = mbar_wait(qfull0 + 8 * slot, (qi / C::kQueue) & 1, &s_abort, a.err);
      const DecodeItem it = *reinterpret_cast<const DecodeItem*>(queue + slot * C::kEntryBytes);
      // every consumer warp leaves at the same item (the named barriers below
      // need every one): the stop decision is OR-reduced over them
      if (consumer_any<C::kWarps>(!got || it.ntok < 0 || s_abort != 0)) break;
      float qf[G][C::kEPV];
      float o[G][C::kEPV];
      float m[G], l[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const uint4 u = *reinterpret_cast<const uint4*>(queue + slot * C::kEntryBytes + 64 + h * C::kRowBytes + c * 16);
        Elem<T>::unpack(u, qf[h]);
#pragma unroll
        for (int e = 0; e < C::kEPV; ++e) qf[h][e] *= a.scale_log2;
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < C::kEPV; ++e) o[h][e] = 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(qempty0 + 8 * slot);  // entry read: the producer may reuse it
      const int ntiles = (it.ntok + C::kTile - 1) / C::kTile;
      for (int t = 0; t < ntiles; ++t, ++g) {
        const uint32_t s = g % C::kStages;
        if (!mbar_wait(full0 + 8 * s, (g / C::kStages) & 1, &s_abort, a.err)) {
          g += ntiles - t;  // keep the ring position consistent (the kernel is ending anyway)
          break;
        }
        const uint8_t* tk = sk + s * C::kTileBytes;
        const uint8_t* tv = sv + s * C::kTileBytes;
        const int nvalid = min(C::kTile, it.ntok - t * C::kTile);
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
      // the previous split's counter increment was issued one item ago: by now
      // its result is back, and it says whether this CTA merges that pair
      if (threadIdx.x == 0) publish_pending();
      consumer_sync<C::kWarps>();

      // ---- merge the consumer warps: result for (h, d) of this split
      const int bh = it.b * a.hkv + it.kvh;
      const bool single = (it.nsplit == 1);
      for (int idx = threadIdx.x; idx < G * D; idx += C::kWarps * 32) {
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
        const int qh = it.kvh * G + h;
        if (single) {
          pair_result<T, D, XCHG>(a, it.b, qh, d, ov, lse, xpar);
        } else {
          a.ws_o[(((int64_t)bh * a.max_splits + it.split) * G + h) * D + d] = ov;
          if (d == 0) a.ws_lse[((int64_t)bh * a.max_splits + it.split) * G + h] = lse;
        }
      }
      if (s_merge[0]) merge_splits<T, D, G, C::kWarps * 32, XCHG>(a, s_merge[1], s_merge[2], s_merge[3], xpar);
      // the reductions buffer and s_merge are reused by the next item; for a
      // split this barrier also orders the CTA's partial writes before thread
      // 0's acquire-release increment of the pair's split counter at GPU scope
      // (cumulative), which in turn orders every split's partials before the
      // merge that the last increment triggers
      consumer_sync<C::kWarps>();
      if constexpr (XCHG) {
        if (threadIdx.x == 0) {
          if (single) publish_pair(a, bh, xe);
          if (s_merge[0]) publish_pair(a, s_merge[1] * a.hkv + s_merge[2], xe);
        }
      }
      if (!single && threadIdx.x == 0) {
        // issued now, read at the next item's end (or after the last item)
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(pend_prev) : "l"(a.ws_count + bh) : "memory");
        pend_b = it.b;
        pend_kvh = it.kvh;
        pend_nsplit = it.nsplit;
      }
    }
    // ---- the last item's increment: merge its pair if that came last
    if (threadIdx.x == 0) publish_pending();
    consumer_sync<C::kWarps>();
    if (s_merge[0] && s_abort == 0)
      merge_splits<T, D, G, C::kWarps * 32, XCHG>(a, s_merge[1], s_merge[2], s_merge[3], xpar);
    if constexpr (XCHG) {
      // ---- publish that pair, then finalize pairs: merge every rank's result
      const bool merged = s_merge[0] && s_abort == 0;
      consumer_sync<C::kWarps>();
      if (merged && threadIdx.x == 0) publish_pair(a, s_merge[1] * a.hkv + s_merge[2], xe);
      __shared__ int s_fin[2];  // [pair claimed, a peer did not arrive]
      const int pairs = a.batch * a.hkv;
      uint8_t* own = static_cast<uint8_t*>(a.xpeers[a.xrank]);
      const unsigned long long* pflags = reinterpret_cast<const unsigned long long*>(own + kExchangePairFlags);
      const float* slots = reinterpret_cast<const float*>(own + a.xslot_off) + (int64_t)xpar * a.xworld * a.xslot_floats;
      const int64_t n_o = (int64_t)a.batch * a.hq * D;
      for (;;) {
        if (threadIdx.x == 0) {
          s_fin[0] = s_abort ? pairs : (int)atomicAdd(a.ws_sched + 2, 1u);
          s_fin[1] = 0;
        }
        consumer_sync<C::kWarps>();
        const int pair = s_fin[0];
        if (pair >= pairs) break;  // every consumer thread read the same value
        if (threadIdx.x < a.xworld) {
          const unsigned long long t0 = global_timer_ns();
          for (uint32_t it = 1; ld_relaxed_sys(pflags + (int64_t)pair * 8 + threadIdx.x) < xe; ++it) {
            if ((it & 63u) == 0u && global_timer_ns() - t0 > a.xbudget) {
              flag_device_error(a.err, AICAS_DEVERR_PEER_TIMEOUT);
              s_fin[1] = 1;
              break;
            }
          }
          fence_acq_rel_sys();
        }
        consumer_sync<C::kWarps>();
        const int b = pair / a.hkv, kvh = pair % a.hkv;
        for (int idx = threadIdx.x; idx < G * D; idx += C::kWarps * 32) {
          const int h = idx / D, d = idx % D, qh = kvh * G + h;
          const int64_t bh = (int64_t)b * a.hq + qh;
          // L2 reads (this SM's L1 may hold the slot from two calls ago), all
          // ranks' loads issued together
          float lr[kMaxExchangeRanks], orr[kMaxExchangeRanks];
          float M = -INFINITY;
#pragma unroll
          for (int r = 0; r < kMaxExchangeRanks; ++r) {
            const bool in = r < a.xworld && !s_fin[1];
            const float* sr = slots + (int64_t)r * a.xslot_floats;
            lr[r] = in ? __ldcg(sr + n_o + bh) : -INFINITY;
            orr[r] = in ? __ldcg(sr + bh * D + d) : 0.f;
            M = fmaxf(M, lr[r]);
          }
          float L = 0.f, O = 0.f;
          if (M != -INFINITY) {
#pragma unroll
            for (int r = 0; r < kMaxExchangeRanks; ++r) {
              const float w = exp2f(lr[r] - M);  // 0 for ranks past the world
              L += w;
              O = fmaf(w, orr[r], O);
            }
          }
          if (a.out != nullptr)
            static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)qh * a.o_sh + d] = Elem<T>::from_float(L > 0.f ? O / L : 0.f);
          if (a.lse != nullptr && d == 0) a.lse[bh] = L > 0.f ? M + log2f(L) : -INFINITY;
        }
        consumer_sync<C::kWarps>();  // s_fin is reused by the next claim
      }
    }
  }

  // ---- scheduling counters back to zero for the next call: the last CTA out resets them
  if (dynamic) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned int done = atomicAdd(a.ws_sched + 1, 1u);
      if (done == gridDim.x - 1) {
        a.ws_sched[0] = 0u;
        a.ws_sched[1] = 0u;
        if constexpr (XCHG) {
          a.ws_sched[2] = 0u;
          // this call is complete on this rank: every epoch word (one per
          // exchange-kernel CTA) moves, so either kernel can make the next call
          for (int r = 0; r < a.xworld; ++r)
            reinterpret_cast<volatile unsigned long long*>(static_cast<uint8_t*>(a.xpeers[a.xrank]) + 256)[r] = xe;
        }
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------------ host side

template <typename T, int D, int G, bool XCHG>
static cudaError_t launch_decode_t(const DecodeArgs& a, cudaStream_t st) {
  using C = DecodeCfg<T, D, G>;
  // the dynamic shared-memory opt-in and the co-resident CTA count are per
  // function and per device
  static int resident[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int per_device = (dev >= 0 && dev < 64) ? resident[dev] : 0;
  if (per_device == 0) {
    e = cudaFuncSetAttribute(decode_gqa_kernel<T, D, G, XCHG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemBytes);
    if (e != cudaSuccess) return e;
    int per_sm = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_gqa_kernel<T, D, G, XCHG>, C::kThreads,
                                                      C::kSmemBytes);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    per_device = per_sm * sms;
    if (per_device <= 0) return cudaErrorInvalidConfiguration;
    if (dev >= 0 && dev < 64) resident[dev] = per_device;
  }
  const long long items = (long long)a.batch * a.hkv * a.max_splits;
  const int grid = (int)(items < per_device ? items : per_device);
  // the first items' K/V into L2 ahead of the dependency wait, when they fit
  // comfortably (a larger prefetch would evict itself before it is read)
  DecodeArgs b = a;
  const long long first_bytes = (long long)grid * (a.split_tokens < a.cap ? a.split_tokens : a.cap) * 2 * C::kRowBytes;
  b.prefetch_first = (a.ws_sched != nullptr && first_bytes <= (64ll << 20)) ? 1 : 0;
  return launch_pdl(decode_gqa_kernel<T, D, G, XCHG>, dim3(grid), dim3(C::kThreads), C::kSmemBytes, st, b);
}

template <typename T, int D, bool XCHG = false>
static cudaError_t dispatch_g(int g, const DecodeArgs& a, cudaStream_t st) {
  switch (g) {
    case 1: return launch_decode_t<T, D, 1, XCHG>(a, st);
    case 2: return launch_decode_t<T, D, 2, XCHG>(a, st);
    case 4: return launch_decode_t<T, D, 4, XCHG>(a, st);
    case 8: return launch_decode_t<T, D, 8, XCHG>(a, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t dispatch_d(int d, int g, const DecodeArgs& a, cudaStream_t st) {
  switch (d) {
    case 16: return dispatch_g<T, 16>(g, a, st);
    case 32: return dispatch_g<T, 32>(g, a, st);
    case 64: return dispatch_g<T, 64>(g, a, st);
    case 128: return dispatch_g<T, 128>(g, a, st);
  }
  return cudaErrorInvalidValue;
}

// tokens per stage: 16 KB of rows
int decode_tile_for(int dtype, int head_dim) {
  const int elem = dtype == AICAS_DTYPE_F32 ? 4 : 2;
  return 16384 / (head_dim * elem);
}

// The decode with the cross-GPU merge fused in: 16-bit caches at head_dim 128
// (the sequence-sharded long-context decode of Qwen3-VL-2B's text decoder).
cudaError_t launch_decode_exchange(int dtype, int group, const DecodeArgs& a, cudaStream_t st) {
  switch (dtype) {
    case AICAS_DTYPE_F16: return dispatch_g<__half, 128, true>(group, a, st);
    case AICAS_DTYPE_BF16: return dispatch_g<__nv_bfloat16, 128, true>(group, a, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_decode(int dtype, int head_dim, int group, const DecodeArgs& a, cudaStream_t st) {
  switch (dtype) {
    case AICAS_DTYPE_F32: return dispatch_d<float>(head_dim, group, a, st);
    case AICAS_DTYPE_F16: return dispatch_d<__half>(head_dim, group, a, st);
    case AICAS_DTYPE_BF16: return dispatch_d<__nv_bfloat16>(head_dim, group, a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace aicas
