// The vision attention's packed QKV projection with its RoPE in the epilogue,
// on the sm_100a tensor cores.
//
// Qwen3VLVisionAttention.forward (transformers models/qwen3_vl/
// modeling_qwen3_vl.py:205-209) computes qkv = x W^T + b with one nn.Linear,
// splits it into q, k, v of [T, H, D] and rotates q and k with
// apply_rotary_pos_emb_vision (:131-142).  This kernel produces the same packed
// [T, 3, H, D] tensor in one pass over x: the product accumulates in fp32 in
// tensor memory, the epilogue adds the bias and rounds to the dtype (the
// Linear's output), and for the q and k columns rotates each head row as HF
// does (x * cos + rotate_half(x) * sin with every operation rounded in fp32,
// the result once to the dtype).  v is stored as projected.
//
// Persistent, one CTA per SM, warp-specialised:
//   warp 0      TMA producer: x tile 128 x 64 and W tile 256 x 64 per K step
//               (128-byte swizzle) into a 3-stage ring
//   warp 1      TMEM allocator and the single MMA-issuing thread: tcgen05.mma
//               M=128 N=256 K=16, accumulating a 128 x 256 output tile in one of
//               two TMEM buffers (2 x 256 columns)
//   warps 4-11  epilogue (two warpgroups, half of every head's columns
//               each), one output row (TMEM lane) per thread, reading one
//               buffer while the tensor core fills the other; the finished
//               tile is staged in shared memory and written by TMA stores
//               (whole lines, rows past T clipped by the tensor map)
// Tiles go out m-block-major (12 column tiles of one 128-row block one after
// another), so the CTAs working at the same time share their x rows in L2; W
// (6 MB at Qwen3-VL-2B's size) stays in L2.
#include <cstdio>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma_host.cuh"
#include "vision_qkv.cuh"

namespace aicas {
namespace {

constexpr int kQBM = 128;     // token rows per tile
constexpr int kQBN = 256;     // output features per tile (four 64-wide heads)
constexpr int kQBK = 64;      // K per stage (128 bytes of bf16: one swizzle row)
constexpr int kQStages = 3;
constexpr uint32_t kQATile = kQBM * kQBK * 2;   // 16 KB
constexpr uint32_t kQBTile = kQBN * kQBK * 2;   // 32 KB
constexpr uint32_t kQStage = kQATile + kQBTile;  // 48 KB
// the output tile staged for the TMA store: four [128 rows x 64 columns]
// boxes (one per head), 128-byte swizzled rows
constexpr uint32_t kQOutOff = kQStages * kQStage;
constexpr uint32_t kQOutBox = kQBM * 64 * 2;     // 16 KB
constexpr uint32_t kQBarOff = kQOutOff + 4 * kQOutBox;
constexpr int kQNumBars = 2 * kQStages + 4 + 1;  // full, empty, acc_full[2], acc_empty[2], mma_done
constexpr uint32_t kQMisc = kQBarOff + kQNumBars * 8;
constexpr uint32_t kQSmem = kQMisc + 64 + 1024;  // + slack to align the base to 1024
constexpr int kQThreads = 384;  // producer, MMA, 2 idle warps, two epilogue warpgroups

struct VisionQkvArgs {
  CUtensorMap tm_x;  // [T, K], box {64, 128}
  CUtensorMap tm_w;  // [N, K], box {64, 256}
  CUtensorMap tm_o;  // [T, N], box {64, 128}: the store of one head's 64 columns of a tile
  const void* bias;  // [N] or null
  const float* cos;  // [T, D]
  const float* sin;
  int64_t cs_st;
  int tokens, k_steps, n_tiles, m_tiles, rope_cols;  // rope_cols: the first 2*H*D columns are q and k
  unsigned int* err;
};

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return Elem<T>::to_float(Elem<T>::from_float(x));
}

// Named barrier 1 over the two epilogue warpgroups (256 threads), returning
// the OR of their predicates so that all of them take the same branch after it.
__device__ __forceinline__ bool epilogue_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

template <typename T>
__global__ void __launch_bounds__(kQThreads, 1) vision_qkv_kernel(const __grid_constant__ VisionQkvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (sb - raw);
  const uint32_t bar0 = sb + kQBarOff;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (kQStages + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * kQStages + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * kQStages + 2 + b); };
  const uint32_t mma_done = bar0 + 8u * (2 * kQStages + 4);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gb + kQMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gb + kQMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = a.m_tiles * a.n_tiles;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 256);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(sb + kQMisc, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0 && tmem != 0u) {  // the whole of tensor memory: column 0, lane 0
    flag_device_error(a.err, AICAS_DEVERR_TMEM);
    *abort_flag = 1;
  }
  __syncthreads();
  // launched with programmatic dependent launch: x (the previous kernel's
  // output) is read only after this
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && !*abort_flag) {
      tma_prefetch_desc(&a.tm_x);
      tma_prefetch_desc(&a.tm_w);
      uint32_t g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        const int m0 = (tile / a.n_tiles) * kQBM, n0 = (tile % a.n_tiles) * kQBN;
        for (int kb = 0; kb < a.k_steps; ++kb, ++g) {
          const uint32_t s = g % kQStages, u = g / kQStages;
          if (u > 0 && !mbar_wait(empty(s), (u - 1) & 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full(s), kQStage);
          const uint32_t dst = sb + s * kQStage;
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
              "l"(reinterpret_cast<uint64_t>(&a.tm_x)), "r"(kb * kQBK), "r"(m0), "r"(full(s))
              : "memory");
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst + kQATile),
              "l"(reinterpret_cast<uint64_t>(&a.tm_w)), "r"(kb * kQBK), "r"(n0), "r"(full(s))
              : "memory");
        }
      }
      if (!ok || *abort_flag) {  // let our own copies land before the CTA can retire
        for (uint32_t t = g > (uint32_t)kQStages ? g - kQStages : 0u; t < g; ++t)
          mbar_wait(full(t % kQStages), (t / kQStages) & 1, nullptr, a.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (one thread)
    if (lane == 0) {
      constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t kId = tc::idesc_f16(kBF16, kQBM, kQBN, false, false);
      const uint64_t da0 = tc::smem_desc_sw128(sb, 16, 1024);
      const uint64_t db0 = tc::smem_desc_sw128(sb + kQATile, 16, 1024);
      uint32_t g = 0;
      int it = 0;
      bool ok = !*abort_flag;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++it) {
        const int buf = it & 1, use = it >> 1;
        // the epilogue has read this buffer's previous tile out of tensor memory
        if (use > 0 && !mbar_wait(acc_empty(buf), (use - 1) & 1, abort_flag, a.err)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t acc = tmem + buf * kQBN;
        for (int kb = 0; kb < a.k_steps; ++kb, ++g) {
          const uint32_t s = g % kQStages;
          if (!mbar_wait(full(s), (g / kQStages) & 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t da = da0 + ((uint64_t)(s * kQStage) >> 4);
          const uint64_t db = db0 + ((uint64_t)(s * kQStage) >> 4);
#pragma unroll
          for (int kk = 0; kk < kQBK / 16; ++kk)
            tc::mma_f16_ss(acc, da + (uint64_t)((kk * 32) >> 4), db + (uint64_t)((kk * 32) >> 4), kId,
                           (kb > 0 || kk > 0) ? 1u : 0u);
          tc::commit(empty(s));  // the stage is free once these products have read it
        }
        if (!ok) break;
        tc::commit(acc_full(buf));
      }
      // every product issued has completed before the CTA tears down
      tc::commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, a.err);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // warpgroup eg (warps 4-7, 8-11) takes the 8-column groups q = 2 eg and
    // 2 eg + 1 of every head of the tile; a thread owns one row (its TMEM lane):
    // the row's cos/sin of a group are loaded once for the four heads, and each
    // (head, group)'s 8 + 8 accumulator columns (a column and its rotate_half
    // partner 32 apart) come out of tensor memory together
    const int eg = (warp - 4) >> 2;
    const int qw = warp & 3;
    const int r = qw * 32 + lane;  // TMEM lane = row of the tile
    const uint32_t tl = tmem + ((uint32_t)(qw * 32) << 16);
    const T* bias = static_cast<const T*>(a.bias);
    int it = 0;
    bool ok = !*abort_flag;
    const bool issuer = threadIdx.x == 128;  // issues the tile's TMA stores
    uint8_t* stage_row = gb + kQOutOff + r * 128;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1, use = it >> 1;
      const int m0 = (tile / a.n_tiles) * kQBM, n0 = (tile % a.n_tiles) * kQBN;
      // the previous tile's stores have read the staging buffer (the bar.sync
      // below carries that to every epilogue thread); every epilogue thread
      // takes the same path through these barriers
      if (issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full(buf), use & 1, abort_flag, a.err));
      if (epilogue_any(!got)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int row = m0 + r;
      const bool live = row < a.tokens;
      const bool rope = n0 < a.rope_cols;
      const float* cs = a.cos + (int64_t)row * a.cs_st;
      const float* sn = a.sin + (int64_t)row * a.cs_st;
#pragma unroll 1
      for (int qi = 0; qi < 2; ++qi) {
        const int q = 2 * eg + qi;
        // accumulator columns [h*64 + 8q, +8) and [h*64 + 32 + 8q, +8) of the four heads
        uint32_t acc[4][16];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint32_t col = buf * kQBN + h * 64 + 8 * q;
          tc::tmem_ld8(tl + col, acc[h]);
          tc::tmem_ld8(tl + col + 32, acc[h] + 8);
        }
        tc::tmem_wait_ld();
        if (qi == 1) {
          // this thread's part of the tile is in registers: it releases the buffer
          tc::fence_before_sync();
          mbar_arrive(acc_empty(buf));
        }
        if (!live) continue;
        float c1[8], c2[8], s1[8], s2[8];
        if (rope) {
#pragma unroll
          for (int e = 0; e < 8; e += 4) {
            *reinterpret_cast<float4*>(c1 + e) = __ldg(reinterpret_cast<const float4*>(cs + 8 * q + e));
            *reinterpret_cast<float4*>(c2 + e) = __ldg(reinterpret_cast<const float4*>(cs + 32 + 8 * q + e));
            *reinterpret_cast<float4*>(s1 + e) = __ldg(reinterpret_cast<const float4*>(sn + 8 * q + e));
            *reinterpret_cast<float4*>(s2 + e) = __ldg(reinterpret_cast<const float4*>(sn + 32 + 8 * q + e));
          }
        }
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) {
          const int c0 = hh * 64 + 8 * q;  // column of the tile
          float b1[8], b2[8];
          if (bias != nullptr) {
            Elem<T>::unpack(__ldg(reinterpret_cast<const uint4*>(bias + n0 + c0)), b1);
            Elem<T>::unpack(__ldg(reinterpret_cast<const uint4*>(bias + n0 + c0 + 32)), b2);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) b1[e] = b2[e] = 0.f;
          }
          float y1[8], y2[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            // the Linear's output: fp32 accumulation plus bias, rounded once to the dtype
            y1[e] = round_to<T>(__fadd_rn(__uint_as_float(acc[hh][e]), b1[e]));
            y2[e] = round_to<T>(__fadd_rn(__uint_as_float(acc[hh][8 + e]), b2[e]));
          }
          uint32_t w1[4], w2[4];
          if (rope) {
            // (x * cos) + (rotate_half(x) * sin), each operation rounded in fp32
            float o1[8], o2[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              o1[e] = __fadd_rn(__fmul_rn(y1[e], c1[e]), __fmul_rn(-y2[e], s1[e]));
              o2[e] = __fadd_rn(__fmul_rn(y2[e], c2[e]), __fmul_rn(y1[e], s2[e]));
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              w1[e] = pack_pair<T>(o1[2 * e], o1[2 * e + 1]);
              w2[e] = pack_pair<T>(o2[2 * e], o2[2 * e + 1]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              w1[e] = pack_pair<T>(y1[2 * e], y1[2 * e + 1]);
              w2[e] = pack_pair<T>(y2[2 * e], y2[2 * e + 1]);
            }
          }
          // 16-byte chunks q and q + 4 of this row in head hh's box, XOR-swizzled by row
          uint8_t* box = stage_row + hh * kQOutBox;
          *reinterpret_cast<uint4*>(box + ((q ^ (r & 7)) << 4)) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
          *reinterpret_cast<uint4*>(box + (((q + 4) ^ (r & 7)) << 4)) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
        }
      }
      // the staged tile is visible to the TMA unit, then one thread stores it
      fence_proxy_async_smem();
      epilogue_any(false);
      if (issuer) {
#pragma unroll
        for (int h = 0; h < kQBN / 64; ++h)
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                           reinterpret_cast<uint64_t>(&a.tm_o)),
                       "r"(n0 + h * 64), "r"(m0), "r"(sb + kQOutOff + h * kQOutBox)
                       : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
    }
    // the stores have finished reading shared memory before the CTA can retire
    if (issuer) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }

  // ---------------------------------------------------------------- teardown
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

bool make_map_2d(CUtensorMap* m, const void* ptr, bool bf16, int64_t inner, int64_t rows, int64_t row_stride,
                 int box_rows, char* err, size_t errlen) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (enc == nullptr) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kQBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                         const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (%d) for [%lld, %lld] with row stride %lld", (int)r,
             (long long)rows, (long long)inner, (long long)row_stride);
    return false;
  }
  return true;
}

template <typename T>
cudaError_t launch_qkv(const VisionQkvArgs& a, int grid, cudaStream_t st) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(vision_qkv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kQSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  return launch_pdl(vision_qkv_kernel<T>, dim3(grid), dim3(kQThreads), kQSmem, st, a);
}

}  // namespace

int run_vision_qkv(const aicas_vision_qkv_params* p, int sms, cudaStream_t stream, unsigned int* dev_err, char* err,
                   size_t errlen) {
  const bool bf16 = p->dtype == AICAS_DTYPE_BF16;
  const int n = 3 * p->heads * p->head_dim;
  VisionQkvArgs a;
  memset(&a, 0, sizeof(a));
  if (!make_map_2d(&a.tm_x, p->x, bf16, p->in_features, p->tokens, p->x_stride, kQBM, err, errlen) ||
      !make_map_2d(&a.tm_w, p->weight, bf16, p->in_features, n, p->weight_stride, kQBN, err, errlen) ||
      !make_map_2d(&a.tm_o, p->out, bf16, n, p->tokens, p->out_stride, kQBM, err, errlen))
    return AICAS_ERR_UNSUPPORTED;
  a.bias = p->bias;
  a.cos = p->cos;
  a.sin = p->sin;
  a.cs_st = p->cs_stride_t;
  a.tokens = p->tokens;
  a.k_steps = p->in_features / kQBK;
  a.n_tiles = n / kQBN;
  a.m_tiles = (p->tokens + kQBM - 1) / kQBM;
  a.rope_cols = 2 * p->heads * p->head_dim;
  a.err = dev_err;
  const long long tiles = (long long)a.m_tiles * a.n_tiles;
  const int grid = (int)(tiles < sms ? tiles : sms);
  const cudaError_t e = bf16 ? launch_qkv<__nv_bfloat16>(a, grid, stream) : launch_qkv<__half>(a, grid, stream);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "vision QKV launch: %s (%s)", cudaGetErrorString(e), cudaGetErrorName(e));
    return AICAS_ERR_CUDA;
  }
  return AICAS_OK;
}

}  // namespace aicas
