// C ABI entry points: argument validation, launch planning and error reporting.
// Nothing here allocates device memory or synchronises the device (except the
// one-time peer-buffer set-up calls aicas_peer_buffer_alloc/free, and
// the explicit health query aicas_device_error_flags).
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "fmha.cuh"
#include "linear.cuh"
#include "vision_qkv.cuh"

namespace aicas {

struct DecodeArgs;
cudaError_t launch_decode(int dtype, int head_dim, int group, const DecodeArgs& a, cudaStream_t st);
cudaError_t launch_decode_exchange(int dtype, int group, const DecodeArgs& a, cudaStream_t st);
int decode_tile_for(int dtype, int head_dim);
struct RopeArgs;
cudaError_t launch_rope_append(int dtype, int cs_dtype, const RopeArgs& a, cudaStream_t st);
struct VisionRopeArgs;
cudaError_t launch_vision_rope(int dtype, const VisionRopeArgs& a, int sms, cudaStream_t st);
struct MergeArgs;
cudaError_t launch_merge(int dtype, const MergeArgs& a, cudaStream_t st);
struct ExchangeArgs;
cudaError_t launch_exchange_merge(int dtype, const ExchangeArgs& a, cudaStream_t st);
size_t exchange_slot_floats(int batch, int heads, int head_dim);
size_t exchange_buffer_bytes(int world, int batch, int heads, int head_dim);

}  // namespace aicas

// The full definitions are needed to fill the argument blocks.
#include "args.cuh"

namespace {

// The device error word (AICAS_DEVERR_* bits), one per device context.
__device__ unsigned int g_device_error = 0;

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(AICAS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case AICAS_DTYPE_F32: return 4;
    case AICAS_DTYPE_F16: return 2;
    case AICAS_DTYPE_BF16: return 2;
  }
  return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride_ok(int64_t stride, int eb) { return ((stride * eb) & 15) == 0; }
bool is_pow2_group(int g) { return g == 1 || g == 2 || g == 4 || g == 8; }
bool head_dim_ok(int d) { return d == 16 || d == 32 || d == 64 || d == 128; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// The calling thread's current CUDA context (the driver's cuCtxGetCurrent,
// fetched through the runtime so the library links no driver library); NULL
// before the runtime has made one current.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CUcontext current_context() {
  static const CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// Device addresses of a __device__ array, one per CUDA context: a module's
// globals live at a different address in every context (a host may create
// its own contexts next to the runtime's primary one), so the address is
// looked up once per context, with that context current.
class SymbolAddresses {
 public:
  explicit SymbolAddresses(const void* symbol) : symbol_(symbol) {}
  cudaError_t get(void** out) {
    CUcontext ctx = current_context();
    {
      std::lock_guard<std::mutex> lock(mu_);
      for (int i = 0; i < n_ && ctx != nullptr; ++i)
        if (entries_[i].ctx == ctx) {
          *out = entries_[i].ptr;
          return cudaSuccess;
        }
    }
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, symbol_);
    if (e != cudaSuccess) return e;
    if (ptr == nullptr) return cudaErrorInvalidSymbol;
    if (ctx == nullptr) ctx = current_context();  // the lookup above made the primary context current
    {
      std::lock_guard<std::mutex> lock(mu_);
      if (ctx != nullptr && n_ < kMax) entries_[n_++] = {ctx, ptr};
    }
    *out = ptr;
    return cudaSuccess;
  }

 private:
  static constexpr int kMax = 256;
  struct Entry {
    CUcontext ctx;
    void* ptr;
  };
  const void* symbol_;
  std::mutex mu_;
  Entry entries_[kMax] = {};
  int n_ = 0;
};

// Device address of g_device_error in the current context.
unsigned int* device_error_word() {
  static SymbolAddresses addresses(reinterpret_cast<const void*>(&g_device_error));
  void* ptr = nullptr;
  return addresses.get(&ptr) == cudaSuccess ? static_cast<unsigned int*>(ptr) : nullptr;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Split-KV workspace: [counters: 1 MiB][partial o][partial lse].  The counter
// region holds kMaxSplitUnits split counters and, in its last 64 bytes, the
// persistent kernel's work-item and finished-CTA counters.
constexpr size_t kCounterBytes = (size_t)1 << 20;
constexpr size_t kSchedOffset = kCounterBytes - 64;
constexpr int kMaxSplitUnits = (int)(kSchedOffset / sizeof(unsigned int));

// Split-KV plan shared by aicas_decode_workspace_bytes and aicas_decode_gqa.
struct DecodePlan {
  int split_tokens;
  int split_floor;
  int max_splits;
  size_t ws_o_off, ws_lse_off, ws_count_off, ws_bytes;
};

// compact: with many pairs, take whole caches as items whenever the pairs alone
// balance the CTAs (no workspace then), for callers whose scratch is fixed.
int plan_decode(const aicas_decode_params* p, DecodePlan* out, bool compact = false) {
  const int tile = aicas::decode_tile_for(p->dtype, p->head_dim);
  int split = p->split_tokens;
  int split_floor = 0;
  if (split < 0 || (split > 0 && split % tile != 0))
    return fail(AICAS_ERR_UNSUPPORTED, "split_tokens=%d must be 0 or a positive multiple of %d",
                p->split_tokens, tile);
  if (split == 0) {
    // Persistent CTAs (2 per SM) take the splits as work items.  Every item
    // boundary costs a CTA a few microseconds (partial write, counter, merge),
    // so items are as long as balance allows: with few (request, KV head)
    // pairs, about one item per resident CTA (one wave, no boundaries); with
    // many pairs of ragged lengths, about five items per CTA so that the
    // dynamic hand-out can even out the lengths.
    //
    // In the second case the splits of a cache shrink: split 0 is 1.4x that
    // size (at most half the capacity), the next ones halve down to an eighth
    // of it.  Items are handed out split-major, so the long first splits go
    // first and the short late ones fill in as the CTAs finish, which shortens
    // the tail of the launch (ragged config-2 lengths: ~8 % less time than
    // equal splits).
    const int64_t cap = p->kv_capacity > 0 ? p->kv_capacity : 1;
    const int64_t pairs = (int64_t)p->batch * p->num_kv_heads;
    const int64_t resident = (int64_t)sm_count() * 2;
    const auto round_tiles = [&](int64_t v) {
      v = (v + tile - 1) / tile * tile;
      return v < 4 * tile ? (int64_t)4 * tile : v;
    };
    int64_t s;
    if (2 * pairs <= resident) {
      const int64_t per_pair = resident / pairs;
      s = round_tiles((cap + per_pair - 1) / per_pair);
    } else {
      s = round_tiles((cap * pairs + 5 * resident - 1) / (5 * resident));
      if (s < cap || !compact) {
        const int64_t s0 = std::min(round_tiles(s * 7 / 5), round_tiles(cap / 2));
        split_floor = (int)round_tiles(s0 / 8);
        s = s0;
        if (split_floor >= s) split_floor = 0;  // nothing to halve
      }
    }
    if (s > 16384) s = 16384;
    if (split_floor > s) split_floor = 0;
    split = (int)s;
  }
  const int cap = p->kv_capacity > 0 ? p->kv_capacity : 1;
  out->split_tokens = split;
  out->split_floor = split_floor;
  out->max_splits = aicas::decode_split_count(cap, split, split_floor, tile, /*absorb=*/false);
  const int g = p->num_q_heads / p->num_kv_heads;
  const size_t units = (size_t)p->batch * p->num_kv_heads;
  // the kernel numbers work items (request, KV head, split) with 32-bit ints
  if ((int64_t)units * out->max_splits > (int64_t)INT32_MAX)
    return fail(AICAS_ERR_UNSUPPORTED, "%zu (request, KV head) pairs x %d splits exceed the 2^31 work items of one launch",
                units, out->max_splits);
  if (out->max_splits > 1 && units > kMaxSplitUnits)
    return fail(AICAS_ERR_UNSUPPORTED, "split-KV decode supports at most %d (request, KV head) pairs (got %zu)",
                kMaxSplitUnits, units);
  // Counters live at a FIXED place (the first kCounterBytes) whatever the call's
  // shape, so the zeros one call leaves behind are where the next call, of any
  // shape, looks for them; partial results only ever go after that region.
  size_t off = kCounterBytes;
  out->ws_count_off = 0;
  out->ws_o_off = off;
  off = align_up(off + units * out->max_splits * g * p->head_dim * sizeof(float), 256);
  out->ws_lse_off = off;
  off = align_up(off + units * out->max_splits * g * sizeof(float), 256);
  out->ws_bytes = out->max_splits > 1 ? off : 0;
  return AICAS_OK;
}

int check_decode(const aicas_decode_params* p) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->q == nullptr || p->k == nullptr || p->v == nullptr)
    return fail(AICAS_ERR_INVALID, "q, k and v must be non-NULL");
  if (p->out == nullptr && p->partial_o == nullptr)
    return fail(AICAS_ERR_INVALID, "one of out / partial_o must be set");
  if (p->partial_o != nullptr && p->lse == nullptr)
    return fail(AICAS_ERR_INVALID, "partial_o requires lse");
  const int eb = elem_bytes(p->dtype);
  if (eb == 0) return fail(AICAS_ERR_UNSUPPORTED, "unknown dtype %d", p->dtype);
  if (p->batch < 1 || p->batch > 65535 || p->num_kv_heads < 1 || p->num_kv_heads > 65535 || p->num_q_heads < 1 ||
      p->kv_capacity < 0)
    return fail(AICAS_ERR_INVALID, "batch=%d num_q_heads=%d num_kv_heads=%d kv_capacity=%d", p->batch,
                p->num_q_heads, p->num_kv_heads, p->kv_capacity);
  if (p->num_q_heads % p->num_kv_heads != 0)
    return fail(AICAS_ERR_INVALID, "num_q_heads=%d is not a multiple of num_kv_heads=%d", p->num_q_heads,
                p->num_kv_heads);
  const int g = p->num_q_heads / p->num_kv_heads;
  if (!is_pow2_group(g)) return fail(AICAS_ERR_UNSUPPORTED, "GQA group size %d not in {1,2,4,8}", g);
  if (!head_dim_ok(p->head_dim)) return fail(AICAS_ERR_UNSUPPORTED, "head_dim %d not in {16,32,64,128}", p->head_dim);
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out) || !aligned16(p->partial_o))
    return fail(AICAS_ERR_INVALID, "device pointers must be 16-byte aligned");
  if (!stride_ok(p->q_stride_b, eb) || !stride_ok(p->q_stride_h, eb) || !stride_ok(p->k_stride_b, eb) ||
      !stride_ok(p->k_stride_h, eb) || !stride_ok(p->v_stride_b, eb) || !stride_ok(p->v_stride_h, eb))
    return fail(AICAS_ERR_INVALID, "q/k/v strides must be multiples of 16 bytes");
  if (p->out != nullptr && (p->o_stride_b < 0 || p->o_stride_h < 0))
    return fail(AICAS_ERR_INVALID, "negative output stride");
  if (!(p->sm_scale == p->sm_scale) || p->sm_scale == INFINITY || p->sm_scale == -INFINITY)
    return fail(AICAS_ERR_INVALID, "sm_scale must be finite");
  return AICAS_OK;
}

int check_fmha(const aicas_fmha_params* p, bool varlen) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->q == nullptr || p->k == nullptr || p->v == nullptr || p->out == nullptr)
    return fail(AICAS_ERR_INVALID, "q, k, v and out must be non-NULL");
  if (p->dtype != AICAS_DTYPE_BF16 && p->dtype != AICAS_DTYPE_F16)
    return fail(AICAS_ERR_UNSUPPORTED, "tensor-core attention needs fp16 or bf16 (dtype %d)", p->dtype);
  if (p->head_dim != 64 && p->head_dim != 128)
    return fail(AICAS_ERR_UNSUPPORTED, "tensor-core attention supports head_dim 64 and 128 (got %d)", p->head_dim);
  if (p->batch < 1 || p->num_q_heads < 1 || p->num_kv_heads < 1 || p->seq_len_q < 0 || p->seq_len_kv < 0)
    return fail(AICAS_ERR_INVALID, "bad sizes");
  if (p->num_q_heads % p->num_kv_heads != 0)
    return fail(AICAS_ERR_INVALID, "num_q_heads %% num_kv_heads != 0");
  const int eb = 2;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out))
    return fail(AICAS_ERR_INVALID, "device pointers must be 16-byte aligned");
  const int64_t st[] = {p->q_stride_b, p->q_stride_h, p->q_stride_s, p->k_stride_b, p->k_stride_h, p->k_stride_s,
                        p->v_stride_b, p->v_stride_h, p->v_stride_s, p->o_stride_b, p->o_stride_h, p->o_stride_s};
  for (int64_t s : st)
    if (s < 0 || !stride_ok(s, eb)) return fail(AICAS_ERR_INVALID, "strides must be non-negative multiples of 16 bytes");
  if (!(p->sm_scale == p->sm_scale)) return fail(AICAS_ERR_INVALID, "sm_scale is NaN");
  if (varlen) {
    if (p->batch != 1) return fail(AICAS_ERR_UNSUPPORTED, "varlen attention needs batch == 1");
    if (p->num_q_heads != p->num_kv_heads) return fail(AICAS_ERR_UNSUPPORTED, "varlen attention needs Hq == Hkv");
    if (p->cu_seqlens_q == nullptr || p->cu_seqlens_k == nullptr || p->num_seqs < 0)
      return fail(AICAS_ERR_INVALID, "cu_seqlens_q/k must be set");
    if (p->kv_starts != nullptr) return fail(AICAS_ERR_UNSUPPORTED, "kv_starts applies to causal prefill only");
  } else {
    if (p->seq_len_q != p->seq_len_kv)
      return fail(AICAS_ERR_UNSUPPORTED, "causal prefill needs q_len == kv_len (%d vs %d)", p->seq_len_q, p->seq_len_kv);
  }
  return AICAS_OK;
}

}  // namespace

// Scratch of aicas_decode_gqa_noalloc: split-KV counters (first 1 MiB) and
// partial results, shared by every call of that entry point on a device.
// Zero at module load; each completed call leaves its counters at zero and the
// entry point clears the counters it uses before each launch.
constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Device address of g_noalloc_scratch in the current context.  In host code the
// array's name only stands in for the symbol: the address must be looked up
// (once per context, with that context current) before a kernel may use it.
int noalloc_scratch(void** out) {
  static SymbolAddresses addresses(reinterpret_cast<const void*>(&g_noalloc_scratch));
  const cudaError_t e = addresses.get(out);
  if (e != cudaSuccess)
    return cuda_fail(e, "aicas_decode_gqa_noalloc: cudaGetSymbolAddress of the static scratch");
  return AICAS_OK;
}

}  // namespace

int check_linear(const aicas_linear_params* p) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->dtype != AICAS_DTYPE_F16 && p->dtype != AICAS_DTYPE_BF16)
    return fail(AICAS_ERR_UNSUPPORTED, "decode linear needs fp16 or bf16 (dtype %d)", p->dtype);
  if (p->batch < 0 || p->batch > AICAS_LINEAR_MAX_ROWS)
    return fail(AICAS_ERR_UNSUPPORTED, "decode linear takes 0..%d rows (got %d)", AICAS_LINEAR_MAX_ROWS, p->batch);
  if (p->in_features <= 0 || p->in_features % 8 != 0)
    return fail(AICAS_ERR_UNSUPPORTED, "in_features must be a positive multiple of 8 (got %d)", p->in_features);
  if (p->mode != AICAS_LINEAR_STORE && p->mode != AICAS_LINEAR_RESIDUAL && p->mode != AICAS_LINEAR_SWIGLU)
    return fail(AICAS_ERR_INVALID, "unknown mode %d", p->mode);
  if (p->num_segments < 1 || p->num_segments > AICAS_LINEAR_MAX_SEGMENTS)
    return fail(AICAS_ERR_INVALID, "num_segments must be 1..%d (got %d)", AICAS_LINEAR_MAX_SEGMENTS, p->num_segments);
  if (p->mode == AICAS_LINEAR_RESIDUAL && p->num_segments != 1)
    return fail(AICAS_ERR_INVALID, "the residual epilogue takes one segment");
  if (p->mode == AICAS_LINEAR_SWIGLU && (p->num_segments != 2 || p->seg[0].rows != p->seg[1].rows))
    return fail(AICAS_ERR_INVALID, "the SwiGLU epilogue takes two segments (gate, up) with equal rows");
  if (p->x == nullptr || !aligned16(p->x)) return fail(AICAS_ERR_INVALID, "x must be a 16-byte aligned pointer");
  if (p->x_stride < p->in_features || !stride_ok(p->x_stride, 2))
    return fail(AICAS_ERR_INVALID, "x_stride must be >= in_features and a multiple of 8 elements");
  if (p->norm_weight != nullptr && !aligned16(p->norm_weight))
    return fail(AICAS_ERR_INVALID, "norm_weight must be 16-byte aligned");
  if (p->norm_weight != nullptr && !(p->eps >= 0.0f)) return fail(AICAS_ERR_INVALID, "eps must be >= 0");
  for (int j = 0; j < p->num_segments; ++j) {
    const aicas_linear_segment& g = p->seg[j];
    if (g.weight == nullptr || !aligned16(g.weight))
      return fail(AICAS_ERR_INVALID, "segment %d: weight must be a 16-byte aligned pointer", j);
    if (g.weight_stride < p->in_features || !stride_ok(g.weight_stride, 2))
      return fail(AICAS_ERR_INVALID, "segment %d: weight_stride must be >= in_features and a multiple of 8", j);
    if (g.rows <= 0) return fail(AICAS_ERR_INVALID, "segment %d: rows must be positive", j);
    const bool writes = p->mode != AICAS_LINEAR_SWIGLU || j == 0;
    if (writes && (g.out == nullptr || (reinterpret_cast<uintptr_t>(g.out) & 1u) != 0))
      return fail(AICAS_ERR_INVALID, "segment %d: out must be a 2-byte aligned pointer", j);
    if (writes && p->batch > 1 && g.out_stride < g.rows)
      return fail(AICAS_ERR_INVALID, "segment %d: out_stride must be >= rows", j);
  }
  if (p->sumsq_out != nullptr) {
    if (p->num_segments != 1 || p->mode == AICAS_LINEAR_SWIGLU)
      return fail(AICAS_ERR_INVALID, "sumsq_out takes one segment and a store or residual epilogue");
    if ((reinterpret_cast<uintptr_t>(p->sumsq_out) & 3u) != 0)
      return fail(AICAS_ERR_INVALID, "sumsq_out must be 4-byte aligned");
  }
  if (p->x_sumsq != nullptr) {
    if (p->norm_weight == nullptr) return fail(AICAS_ERR_INVALID, "x_sumsq needs norm_weight");
    if ((reinterpret_cast<uintptr_t>(p->x_sumsq) & 3u) != 0)
      return fail(AICAS_ERR_INVALID, "x_sumsq must be 4-byte aligned");
  }
  if (p->mode == AICAS_LINEAR_RESIDUAL) {
    if (p->residual == nullptr || (reinterpret_cast<uintptr_t>(p->residual) & 1u) != 0)
      return fail(AICAS_ERR_INVALID, "the residual epilogue needs a 2-byte aligned residual");
    if (p->batch > 1 && p->residual_stride < p->seg[0].rows)
      return fail(AICAS_ERR_INVALID, "residual_stride must be >= rows");
  }
  return AICAS_OK;
}

extern "C" {

const char* aicas_version(void) { return "aicas_b200 0.2.0 sm_100a abi 2"; }

uint32_t aicas_capabilities(void) {
  return AICAS_CAP_DECODE | AICAS_CAP_MERGE | AICAS_CAP_ROPE_APPEND | AICAS_CAP_PEER_EXCHANGE |
         AICAS_CAP_DECODE_LINEAR | AICAS_CAP_VISION_ROPE | AICAS_CAP_VISION_QKV | aicas::fmha_capabilities();
}

const char* aicas_last_error(void) { return g_err; }

int aicas_device_error_flags(uint32_t* flags, int clear) {
  if (flags == nullptr) return fail(AICAS_ERR_INVALID, "flags is NULL");
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  *flags = v;
  if (clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  }
  return AICAS_OK;
}

size_t aicas_decode_workspace_bytes(const aicas_decode_params* p) {
  if (check_decode(p) != AICAS_OK) return 0;
  DecodePlan plan;
  if (plan_decode(p, &plan) != AICAS_OK) return 0;
  return plan.ws_bytes;
}

// Launches the decode of a checked call with its plan (with the cross-GPU merge
// fused in when a checked peer group is given).
int run_decode(const aicas_decode_params* p, const DecodePlan& plan, void* workspace, size_t workspace_bytes,
               void* stream, const aicas_peer_group* group = nullptr) {
  if (plan.ws_bytes > 0 && (workspace == nullptr || workspace_bytes < plan.ws_bytes))
    return fail(AICAS_ERR_WORKSPACE, "decode needs %zu bytes of zero-initialised workspace (got %zu)", plan.ws_bytes,
                workspace_bytes);
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(AICAS_ERR_INVALID, "workspace must be 256-byte aligned");
  aicas::DecodeArgs a;
  a.q = p->q; a.k = p->k; a.v = p->v; a.out = p->out; a.lse = p->lse; a.partial_o = p->partial_o;
  a.kv_lens = p->kv_lens;
  a.kv_starts = p->kv_starts;
  a.q_sb = p->q_stride_b; a.q_sh = p->q_stride_h;
  a.k_sb = p->k_stride_b; a.k_sh = p->k_stride_h;
  a.v_sb = p->v_stride_b; a.v_sh = p->v_stride_h;
  a.o_sb = p->o_stride_b; a.o_sh = p->o_stride_h;
  a.batch = p->batch; a.hq = p->num_q_heads; a.hkv = p->num_kv_heads; a.cap = p->kv_capacity;
  a.scale_log2 = p->sm_scale * 1.4426950408889634f;
  a.split_tokens = plan.split_tokens;
  a.split_floor = plan.split_floor;
  a.max_splits = plan.max_splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.ws_o = plan.ws_bytes ? reinterpret_cast<float*>(ws + plan.ws_o_off) : nullptr;
  a.ws_lse = plan.ws_bytes ? reinterpret_cast<float*>(ws + plan.ws_lse_off) : nullptr;
  a.ws_count = plan.ws_bytes ? reinterpret_cast<unsigned int*>(ws + plan.ws_count_off) : nullptr;
  a.ws_sched = plan.ws_bytes ? reinterpret_cast<unsigned int*>(ws + kSchedOffset) : nullptr;
  a.err = device_error_word();
  memset(a.xpeers, 0, sizeof(a.xpeers));
  a.xworld = a.xrank = 0;
  a.xslot_floats = a.xslot_off = 0;
  a.xbudget = 0;
  cudaError_t e;
  if (group != nullptr) {
    for (int r = 0; r < group->world; ++r) a.xpeers[r] = group->peers[r];
    a.xworld = group->world;
    a.xrank = group->rank;
    a.xslot_floats = (long long)aicas::exchange_slot_floats(p->batch, p->num_q_heads, p->head_dim);
    a.xslot_off = aicas::exchange_slots_offset(p->batch, p->num_q_heads);
    a.xbudget = group->wait_budget_ns != 0 ? group->wait_budget_ns : aicas::kWaitBudgetNs;
    // the finalize phase claims pairs from the schedule counters, which every plan has here
    a.ws_sched = reinterpret_cast<unsigned int*>(ws + kSchedOffset);
    a.ws_count = reinterpret_cast<unsigned int*>(ws + plan.ws_count_off);
    e = aicas::launch_decode_exchange(p->dtype, p->num_q_heads / p->num_kv_heads, a,
                                      static_cast<cudaStream_t>(stream));
  } else {
    e = aicas::launch_decode(p->dtype, p->head_dim, p->num_q_heads / p->num_kv_heads, a,
                             static_cast<cudaStream_t>(stream));
  }
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return AICAS_OK;
}

int aicas_decode_gqa(const aicas_decode_params* p, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_decode(p);
  if (rc != AICAS_OK) return rc;
  DecodePlan plan;
  rc = plan_decode(p, &plan);
  if (rc != AICAS_OK) return rc;
  return run_decode(p, plan, workspace, workspace_bytes, stream);
}

int aicas_decode_gqa_noalloc(const aicas_decode_params* p, void* stream) {
  int rc = check_decode(p);
  if (rc != AICAS_OK) return rc;
  DecodePlan plan;
  rc = plan_decode(p, &plan);
  if (rc != AICAS_OK) return rc;
  if (plan.ws_bytes > kNoAllocScratchBytes && p->split_tokens == 0) {
    // the automatic split table needs more slots than the static scratch has:
    // whole caches as items where the pairs balance the CTAs on their own
    rc = plan_decode(p, &plan, /*compact=*/true);
    if (rc != AICAS_OK) return rc;
  }
  if (plan.ws_bytes > kNoAllocScratchBytes)
    return fail(AICAS_ERR_UNSUPPORTED,
                "aicas_decode_gqa_noalloc: this call needs %zu bytes of split-KV scratch but the library's static "
                "scratch holds %zu; raise split_tokens (fewer splits) or call aicas_decode_gqa with a workspace",
                plan.ws_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (plan.ws_bytes > 0) {
    rc = noalloc_scratch(&scratch);
    if (rc != AICAS_OK) return rc;
    // the split counters of this call must start at zero: clear them (a call
    // that was cut short could have left some behind); partials need no clearing
    const size_t counter_bytes = (size_t)p->batch * p->num_kv_heads * sizeof(unsigned int);
    cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + plan.ws_count_off, 0, counter_bytes,
                                    static_cast<cudaStream_t>(stream));
    // and so must the work-item counters of the persistent kernel
    if (e == cudaSuccess)
      e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + kSchedOffset, 0, 64, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "aicas_decode_gqa_noalloc: clearing the split counters");
  }
  return run_decode(p, plan, scratch, scratch != nullptr ? kNoAllocScratchBytes : 0, stream);
}

int aicas_merge_partials(const aicas_merge_params* p, void* stream) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->partial_o == nullptr || p->partial_lse == nullptr || p->out == nullptr)
    return fail(AICAS_ERR_INVALID, "partial_o, partial_lse and out must be non-NULL");
  if (elem_bytes(p->dtype) == 0) return fail(AICAS_ERR_UNSUPPORTED, "unknown dtype %d", p->dtype);
  if (p->num_partials < 1 || p->batch < 1 || p->num_heads < 1 || p->head_dim < 1 || p->head_dim > 1024)
    return fail(AICAS_ERR_INVALID, "bad sizes");
  aicas::MergeArgs a;
  a.po = p->partial_o; a.plse = p->partial_lse; a.out = p->out; a.lse = p->lse;
  a.o_sb = p->o_stride_b; a.o_sh = p->o_stride_h;
  a.np = p->num_partials; a.batch = p->batch; a.heads = p->num_heads; a.hd = p->head_dim;
  cudaError_t e = aicas::launch_merge(p->dtype, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return AICAS_OK;
}

size_t aicas_exchange_buffer_bytes(int32_t world, int32_t batch, int32_t num_heads, int32_t head_dim) {
  if (world < 1 || world > AICAS_MAX_EXCHANGE_RANKS || batch < 1 || num_heads < 1 || head_dim < 1) return 0;
  return aicas::exchange_buffer_bytes(world, batch, num_heads, head_dim);
}

int aicas_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes == 0)
    return fail(AICAS_ERR_INVALID, "ptr, ipc_handle and a non-zero size are required");
  static_assert(sizeof(cudaIpcMemHandle_t) == AICAS_IPC_HANDLE_BYTES, "IPC handle size");
  *ptr = nullptr;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "aicas_peer_buffer_alloc: cudaMalloc");
  e = cudaMemset(d, 0, bytes);  // flags and epoch start at zero
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, d);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "aicas_peer_buffer_alloc: zeroing / IPC handle");
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = d;
  return AICAS_OK;
}

int aicas_peer_buffer_free(void* ptr) {
  if (ptr == nullptr) return AICAS_OK;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? AICAS_OK : cuda_fail(e, "aicas_peer_buffer_free");
}

int aicas_peer_buffer_open(const void* ipc_handle, void** ptr) {
  if (ptr == nullptr || ipc_handle == nullptr) return fail(AICAS_ERR_INVALID, "ipc_handle and ptr are required");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  *ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? AICAS_OK : cuda_fail(e, "aicas_peer_buffer_open: cudaIpcOpenMemHandle");
}

int aicas_peer_buffer_close(void* ptr) {
  if (ptr == nullptr) return AICAS_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? AICAS_OK : cuda_fail(e, "aicas_peer_buffer_close");
}

int aicas_exchange_merge(const aicas_exchange_params* p, void* stream) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->world < 1 || p->world > AICAS_MAX_EXCHANGE_RANKS || p->rank < 0 || p->rank >= p->world)
    return fail(AICAS_ERR_INVALID, "rank %d of world %d (at most %d ranks)", p->rank, p->world,
                AICAS_MAX_EXCHANGE_RANKS);
  if (p->partial_o == nullptr || p->partial_lse == nullptr || p->out == nullptr)
    return fail(AICAS_ERR_INVALID, "partial_o, partial_lse and out must be non-NULL");
  for (int r = 0; r < p->world; ++r)
    if (p->peers[r] == nullptr || (reinterpret_cast<uintptr_t>(p->peers[r]) & 255u) != 0)
      return fail(AICAS_ERR_INVALID, "exchange buffer of rank %d is NULL or not 256-byte aligned", r);
  if (elem_bytes(p->dtype) == 0) return fail(AICAS_ERR_UNSUPPORTED, "unknown dtype %d", p->dtype);
  if (p->batch < 1 || p->num_heads < 1 || p->head_dim < 4 || p->head_dim > 1024 || (p->head_dim & 3))
    return fail(AICAS_ERR_INVALID, "bad sizes (head_dim must be a multiple of 4)");
  if ((reinterpret_cast<uintptr_t>(p->partial_o) & 15u) != 0)
    return fail(AICAS_ERR_INVALID, "partial_o must be 16-byte aligned");
  {
    const int64_t eb = elem_bytes(p->dtype);
    if ((reinterpret_cast<uintptr_t>(p->out) & 15u) != 0 || (p->o_stride_b * eb) % 16 != 0 || (p->o_stride_h * eb) % 16 != 0)
      return fail(AICAS_ERR_INVALID, "out must be 16-byte aligned with strides that are multiples of 16 bytes");
  }
  aicas::ExchangeArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < p->world; ++r) a.peers[r] = p->peers[r];
  a.po = p->partial_o;
  a.plse = p->partial_lse;
  a.out = p->out;
  a.lse = p->lse;
  a.o_sb = p->o_stride_b;
  a.o_sh = p->o_stride_h;
  a.world = p->world;
  a.rank = p->rank;
  a.batch = p->batch;
  a.heads = p->num_heads;
  a.hd = p->head_dim;
  a.slot_floats = (int)aicas::exchange_slot_floats(p->batch, p->num_heads, p->head_dim);
  a.slot_off = aicas::exchange_slots_offset(p->batch, p->num_heads);
  a.wait_budget_ns = p->wait_budget_ns != 0 ? p->wait_budget_ns : aicas::kWaitBudgetNs;
  a.err = device_error_word();
  const cudaError_t e = aicas::launch_exchange_merge(p->dtype, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "exchange merge launch");
  return AICAS_OK;
}

size_t aicas_decode_exchange_workspace_bytes(const aicas_decode_params* p) {
  if (check_decode(p) != AICAS_OK) return 0;
  DecodePlan plan;
  if (plan_decode(p, &plan) != AICAS_OK) return 0;
  return std::max(plan.ws_bytes, kCounterBytes);
}

int aicas_decode_gqa_exchange(const aicas_decode_params* p, const aicas_peer_group* group, void* workspace,
                              size_t workspace_bytes, void* stream) {
  int rc = check_decode(p);
  if (rc != AICAS_OK) return rc;
  if (group == nullptr) return fail(AICAS_ERR_INVALID, "group is NULL");
  if (group->world < 1 || group->world > AICAS_MAX_EXCHANGE_RANKS || group->rank < 0 || group->rank >= group->world)
    return fail(AICAS_ERR_INVALID, "rank %d of world %d (at most %d ranks)", group->rank, group->world,
                AICAS_MAX_EXCHANGE_RANKS);
  for (int r = 0; r < group->world; ++r)
    if (group->peers[r] == nullptr || (reinterpret_cast<uintptr_t>(group->peers[r]) & 255u) != 0)
      return fail(AICAS_ERR_INVALID, "exchange buffer of rank %d is NULL or not 256-byte aligned", r);
  if (p->out == nullptr || p->partial_o != nullptr)
    return fail(AICAS_ERR_INVALID, "the fused exchange writes the merged out (and lse): out must be set, partial_o NULL");
  if (p->head_dim != 128 || (p->dtype != AICAS_DTYPE_F16 && p->dtype != AICAS_DTYPE_BF16))
    return fail(AICAS_ERR_UNSUPPORTED, "the fused exchange takes 16-bit caches with head_dim 128 (got dtype %d, %d)",
                p->dtype, p->head_dim);
  DecodePlan plan;
  rc = plan_decode(p, &plan);
  if (rc != AICAS_OK) return rc;
  const size_t need = std::max(plan.ws_bytes, kCounterBytes);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(AICAS_ERR_WORKSPACE, "the fused exchange needs %zu bytes of zero-initialised workspace (got %zu)", need,
                workspace_bytes);
  return run_decode(p, plan, workspace, workspace_bytes, stream, group);
}

int aicas_rope_kv_append(const aicas_rope_append_params* p, void* stream) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->q_in == nullptr || p->q_out == nullptr || p->k_in == nullptr || p->v_in == nullptr || p->cos == nullptr ||
      p->sin == nullptr || p->k_cache == nullptr || p->v_cache == nullptr || p->positions == nullptr)
    return fail(AICAS_ERR_INVALID, "q_in, q_out, k_in, v_in, cos, sin, k_cache, v_cache and positions must be set");
  if (elem_bytes(p->dtype) == 0) return fail(AICAS_ERR_UNSUPPORTED, "unknown dtype %d", p->dtype);
  if (p->cs_dtype != p->dtype && p->cs_dtype != AICAS_DTYPE_F32)
    return fail(AICAS_ERR_UNSUPPORTED, "cos/sin dtype must equal the tensor dtype or be fp32");
  if (p->head_dim < 2 || p->head_dim > 128 || (p->head_dim & 1))
    return fail(AICAS_ERR_UNSUPPORTED, "head_dim must be even and <= 128 (got %d)", p->head_dim);
  if (p->batch < 1 || p->num_q_heads < 1 || p->num_kv_heads < 1 || p->seq_len < 1 || p->capacity < 0)
    return fail(AICAS_ERR_INVALID, "bad sizes");
  aicas::RopeArgs a;
  a.q_in = p->q_in; a.q_out = p->q_out; a.k_in = p->k_in; a.v_in = p->v_in; a.cos = p->cos; a.sin = p->sin;
  a.k_cache = p->k_cache; a.v_cache = p->v_cache; a.positions = p->positions; a.kv_lens_out = p->kv_lens_out;
  a.qw = p->q_norm_weight; a.kw = p->k_norm_weight; a.eps = p->norm_eps;
  a.qi_sb = p->qi_stride_b; a.qi_sh = p->qi_stride_h; a.qi_ss = p->qi_stride_s;
  a.qo_sb = p->qo_stride_b; a.qo_sh = p->qo_stride_h; a.qo_ss = p->qo_stride_s;
  a.k_sb = p->k_stride_b; a.k_sh = p->k_stride_h; a.k_ss = p->k_stride_s;
  a.v_sb = p->v_stride_b; a.v_sh = p->v_stride_h; a.v_ss = p->v_stride_s;
  a.cs_sb = p->cs_stride_b; a.cs_ss = p->cs_stride_s;
  a.kc_sb = p->kc_stride_b; a.kc_sh = p->kc_stride_h; a.vc_sb = p->vc_stride_b; a.vc_sh = p->vc_stride_h;
  a.batch = p->batch; a.hq = p->num_q_heads; a.hkv = p->num_kv_heads; a.seq = p->seq_len; a.hd = p->head_dim;
  a.cap = p->capacity;
  cudaError_t e = aicas::launch_rope_append(p->dtype, p->cs_dtype, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope/append launch");
  return AICAS_OK;
}

int aicas_prefill_gqa_causal(const aicas_fmha_params* p, void* stream) {
  int rc = check_fmha(p, false);
  if (rc != AICAS_OK) return rc;
  return aicas::run_fmha(p, /*varlen=*/false, static_cast<cudaStream_t>(stream), device_error_word(), g_err, sizeof(g_err));
}

int aicas_varlen_attention(const aicas_fmha_params* p, void* stream) {
  int rc = check_fmha(p, true);
  if (rc != AICAS_OK) return rc;
  return aicas::run_fmha(p, /*varlen=*/true, static_cast<cudaStream_t>(stream), device_error_word(), g_err, sizeof(g_err));
}

int aicas_vision_rope(const aicas_vision_rope_params* p, void* stream) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->dtype != AICAS_DTYPE_F16 && p->dtype != AICAS_DTYPE_BF16)
    return fail(AICAS_ERR_UNSUPPORTED, "vision RoPE needs fp16 or bf16 q/k (dtype %d)", p->dtype);
  if (p->tokens < 0 || p->heads <= 0 || p->head_dim <= 0)
    return fail(AICAS_ERR_INVALID, "tokens=%d heads=%d head_dim=%d", p->tokens, p->heads, p->head_dim);
  if (p->head_dim % 16 != 0 || p->head_dim > 256)
    return fail(AICAS_ERR_UNSUPPORTED, "vision RoPE needs head_dim a multiple of 16 up to 256 (got %d)", p->head_dim);
  if (p->tokens == 0) return AICAS_OK;
  if (p->q_in == nullptr || p->k_in == nullptr || p->q_out == nullptr || p->k_out == nullptr || p->cos == nullptr ||
      p->sin == nullptr)
    return fail(AICAS_ERR_INVALID, "q_in, k_in, q_out, k_out, cos and sin must be set");
  if (!aligned16(p->q_in) || !aligned16(p->k_in) || !aligned16(p->q_out) || !aligned16(p->k_out) ||
      !aligned16(p->cos) || !aligned16(p->sin))
    return fail(AICAS_ERR_INVALID, "device pointers must be 16-byte aligned");
  const int64_t st16[] = {p->qi_stride_t, p->qi_stride_h, p->ki_stride_t, p->ki_stride_h,
                          p->qo_stride_t, p->qo_stride_h, p->ko_stride_t, p->ko_stride_h};
  for (int64_t s : st16)
    if (s < 0 || !stride_ok(s, 2)) return fail(AICAS_ERR_INVALID, "q/k strides must be non-negative multiples of 8");
  if (p->cs_stride_t < p->head_dim || (p->cs_stride_t & 3) != 0)
    return fail(AICAS_ERR_INVALID, "cos/sin row stride must be >= head_dim and a multiple of 4");
  aicas::VisionRopeArgs a;
  a.q_in = p->q_in;
  a.k_in = p->k_in;
  a.q_out = p->q_out;
  a.k_out = p->k_out;
  a.cos = p->cos;
  a.sin = p->sin;
  a.qi_st = p->qi_stride_t;
  a.qi_sh = p->qi_stride_h;
  a.ki_st = p->ki_stride_t;
  a.ki_sh = p->ki_stride_h;
  a.qo_st = p->qo_stride_t;
  a.qo_sh = p->qo_stride_h;
  a.ko_st = p->ko_stride_t;
  a.ko_sh = p->ko_stride_h;
  a.cs_st = p->cs_stride_t;
  a.tokens = p->tokens;
  a.heads = p->heads;
  a.hd = p->head_dim;
  const cudaError_t e = aicas::launch_vision_rope(p->dtype, a, sm_count(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vision RoPE launch");
  return AICAS_OK;
}

int aicas_vision_qkv_rope(const aicas_vision_qkv_params* p, void* stream) {
  if (p == nullptr) return fail(AICAS_ERR_INVALID, "params is NULL");
  if (p->dtype != AICAS_DTYPE_F16 && p->dtype != AICAS_DTYPE_BF16)
    return fail(AICAS_ERR_UNSUPPORTED, "vision QKV needs fp16 or bf16 (dtype %d)", p->dtype);
  if (p->tokens < 0 || p->heads <= 0 || p->in_features <= 0)
    return fail(AICAS_ERR_INVALID, "tokens=%d heads=%d in_features=%d", p->tokens, p->heads, p->in_features);
  if (p->head_dim != 64 || p->heads % 4 != 0)
    return fail(AICAS_ERR_UNSUPPORTED, "vision QKV needs head_dim 64 and a multiple of 4 heads (got %d, %d)",
                p->head_dim, p->heads);
  if (p->in_features % 64 != 0)
    return fail(AICAS_ERR_UNSUPPORTED, "vision QKV needs in_features a multiple of 64 (got %d)", p->in_features);
  if (p->tokens == 0) return AICAS_OK;
  const int64_t n = 3LL * p->heads * p->head_dim;
  if (p->x == nullptr || p->weight == nullptr || p->out == nullptr || p->cos == nullptr || p->sin == nullptr)
    return fail(AICAS_ERR_INVALID, "x, weight, out, cos and sin must be set");
  if (!aligned16(p->x) || !aligned16(p->weight) || !aligned16(p->out) || !aligned16(p->cos) || !aligned16(p->sin))
    return fail(AICAS_ERR_INVALID, "device pointers must be 16-byte aligned");
  if (p->bias != nullptr && !aligned16(p->bias)) return fail(AICAS_ERR_INVALID, "bias must be 16-byte aligned");
  if (p->x_stride < p->in_features || !stride_ok(p->x_stride, 2) || p->weight_stride < p->in_features ||
      !stride_ok(p->weight_stride, 2))
    return fail(AICAS_ERR_INVALID, "x/weight strides must be >= in_features and multiples of 8 elements");
  if (p->out_stride < n || !stride_ok(p->out_stride, 2))
    return fail(AICAS_ERR_INVALID, "out_stride must be >= 3 * heads * head_dim and a multiple of 8");
  if (p->cs_stride_t < p->head_dim || (p->cs_stride_t & 3) != 0)
    return fail(AICAS_ERR_INVALID, "cos/sin row stride must be >= head_dim and a multiple of 4");
  return aicas::run_vision_qkv(p, sm_count(), static_cast<cudaStream_t>(stream), device_error_word(), g_err,
                               sizeof(g_err));
}

size_t aicas_linear_workspace_bytes(const aicas_linear_params* p) {
  if (check_linear(p) != AICAS_OK) return 0;
  size_t bytes = 0;
  if (aicas::plan_linear_workspace(p, sm_count(), &bytes, g_err, sizeof(g_err)) != AICAS_OK) return 0;
  return bytes;
}

int aicas_decode_linear(const aicas_linear_params* p, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_linear(p);
  if (rc != AICAS_OK) return rc;
  return aicas::run_linear(p, sm_count(), workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                           device_error_word(), g_err, sizeof(g_err));
}

}  // extern "C"
