// Argument blocks passed by value to the kernels (host-filled from the C ABI
// parameter structs after validation).
#pragma once
#include <stdint.h>

namespace aicas {

#if defined(__CUDACC__)
#define AICAS_HD __host__ __device__ __forceinline__
#else
#define AICAS_HD inline
#endif

// Split-KV table of the decode kernel, shared by the host plan (workspace size)
// and the kernel (each item's token range).  split_floor == 0: every split
// holds split_tokens tokens.  split_floor > 0: a halving table, split 0 holds
// split_tokens tokens and split s >= 1 holds split_tokens >> s rounded up to
// whole tiles, never fewer than split_floor; the splits handed out last are
// then the short ones, which evens out when the CTAs finish.
AICAS_HD int decode_split_size(int s, int split_tokens, int split_floor, int tile) {
  if (split_floor == 0 || s == 0) return split_tokens;
  const int h = s < 30 ? (split_tokens >> s) : 0;
  const int r = (h + tile - 1) / tile * tile;
  return r > split_floor ? r : split_floor;
}
AICAS_HD int decode_split_start(int s, int split_tokens, int split_floor, int tile) {
  if (split_floor == 0) return s * split_tokens;
  int t = 0;
  for (int i = 0; i < s; ++i) t += decode_split_size(i, split_tokens, split_floor, tile);
  return t;
}
// Number of splits of a cache of len tokens (at least one).  In the halving
// table a last split that would hold fewer than split_floor tokens is folded
// into the split before it (absorb), which then runs to len: a cache just past
// a split boundary costs no extra item.  Without absorb: the table's own count,
// an upper bound for every len up to this one (the workspace's slot count).
AICAS_HD int decode_split_count(int len, int split_tokens, int split_floor, int tile, bool absorb = true) {
  if (split_floor == 0) return len <= split_tokens ? 1 : (len + split_tokens - 1) / split_tokens;
  int t = 0, n = 0;
  do {
    t += decode_split_size(n, split_tokens, split_floor, tile);
    ++n;
  } while (t < len);
  if (absorb && n > 1 && len - (t - decode_split_size(n - 1, split_tokens, split_floor, tile)) < split_floor) --n;
  return n;
}

struct DecodeArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* lse;
  float* partial_o;
  const int32_t* kv_lens;
  const int32_t* kv_starts;  // optional: first valid slot per request (left padding)
  int64_t q_sb, q_sh, k_sb, k_sh, v_sb, v_sh, o_sb, o_sh;
  int batch, hq, hkv, cap;
  float scale_log2;
  int split_tokens;       // tokens of split 0 (of every split when split_floor == 0)
  int split_floor;        // 0: fixed splits; > 0: halving table (decode_split_size)
  int max_splits;
  float* ws_o;            // [B*Hkv, max_splits, G, D]
  float* ws_lse;          // [B*Hkv, max_splits, G]
  unsigned int* ws_count; // [B*Hkv] split counters (null: no split-KV workspace)
  unsigned int* ws_sched; // [2] work-item counter, finished-CTA counter (with a workspace)
  int prefetch_first;     // 1: each CTA brings its first item's K/V range into L2 before the dependency wait
  unsigned int* err;      // device error word
  // the cross-GPU merge fused into the decode (decode_gqa_kernel<..., true>):
  // every rank's exchange buffer as mapped here (see exchange.cu for the layout)
  void* xpeers[8];
  int xworld, xrank;
  long long xslot_floats;       // floats per (parity, source rank) slot
  long long xslot_off;          // byte offset of the slots in a buffer
  unsigned long long xbudget;   // bound of a wait for the peers, ns
};

// Exchange buffer layout, shared by the exchange kernel and the fused decode:
//   [0, 256)      uint64 flags[32]: flags[src] = last epoch rank src published here
//   [256, 320)    uint64 epoch[8]: calls completed by the owner, one word per
//                 exchange-kernel CTA (the fused decode reads word 0 and
//                 advances the first `world` words)
//   [512, slots)  uint64 pair_flags[B * H][8]: [pair][src] = last epoch rank src
//                 published that (request, KV head) pair's partial here (fused decode)
//   [slots, ...)  fp32 slots[2][world][slot_floats]: each source rank's (out, lse)
//                 partial, double-buffered by epoch parity
constexpr long long kExchangePairFlags = 512;
AICAS_HD long long exchange_slots_offset(int batch, int heads) {
  return (kExchangePairFlags + (long long)batch * heads * 8 * 8 + 255) / 256 * 256;
}

struct VisionRopeArgs {
  const void* q_in;
  const void* k_in;
  void* q_out;
  void* k_out;
  const float* cos;  // [T, D] fp32
  const float* sin;
  int64_t qi_st, qi_sh, ki_st, ki_sh, qo_st, qo_sh, ko_st, ko_sh, cs_st;
  int tokens, heads, hd;
};

struct RopeArgs {
  const void* q_in;
  void* q_out;
  const void* k_in;
  const void* v_in;
  const void* cos;
  const void* sin;
  void* k_cache;
  void* v_cache;
  const int32_t* positions;
  int32_t* kv_lens_out;
  const void* qw;
  const void* kw;
  float eps;
  int64_t qi_sb, qi_sh, qi_ss, qo_sb, qo_sh, qo_ss;
  int64_t k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;
  int64_t cs_sb, cs_ss;
  int64_t kc_sb, kc_sh, vc_sb, vc_sh;
  int batch, hq, hkv, seq, hd, cap;
};

constexpr int kMaxExchangeRanks = 8;

struct ExchangeArgs {
  void* peers[kMaxExchangeRanks];  // every rank's exchange buffer, mapped into this device
  const float* po;                 // local partial [B*H*D] fp32
  const float* plse;               // local partial LSE [B*H] fp32 (base 2)
  void* out;
  float* lse;
  int64_t o_sb, o_sh;
  int world, rank, batch, heads, hd;
  int slot_floats;
  long long slot_off;              // byte offset of the slots in a buffer
  unsigned long long wait_budget_ns;  // give up on the peers after this long
  unsigned int* err;               // device error word
};

struct MergeArgs {
  const float* po;
  const float* plse;
  void* out;
  float* lse;
  int64_t o_sb, o_sh;
  int np, batch, heads, hd;
};

}  // namespace aicas
