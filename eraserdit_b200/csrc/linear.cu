// Linear layer y = x W^T + b on the sm_100a tensor cores: BF16 (or E4M3)
// operands, FP32 accumulation in TMEM, bias added in FP32, BF16 output.
//
// Replaces the nn.Linear products of the reference's self-attention path:
// the Q/K/V projections attn.to_q/to_k/to_v (models/dits/eraserdit_attention.py:
// 248-253; nn.Linear(2048, 2048, bias=True), models/dits/eraserdit_transformer.py:
// 253-263), run here as one product over the concatenated weights, and the
// output projection to_out[0] (models/dits/eraserdit_attention.py:216-229).
// The E4M3 instantiation (kind::f8f6f4, K = 32 per product, a per-column
// scale in the epilogue) replaces the scaled_mm products of the FP8 shared
// QKV projection (layers/quantization/qkv_fp8.py:29-63).
//
// Design: a persistent kernel, one CTA per SM, walking 256 x 256 (or, for
// problems with few tiles, 128 x 256) output tiles row-block major, so the
// CTAs running at the same time share their rows of x and the whole weight
// through L2.
//   warp 0      TMA producer: 256 (128) x 64 tiles of x, 256 x 64 of W, through a ring of
//               shared-memory stages (128-byte swizzle, K-major).
//   warp 1      MMA issuer (one thread): two M=128 N=256 accumulators per tile
//               (rows 0-127 and 128-255), K=16 per instruction, TMEM columns
//               [0,256) and [256,512); with 128-row tiles one accumulator in
//               each half of TMEM, alternating between tiles.
//   warps 2-9   epilogue: each warp drains 32 rows x 256 (128) columns of one
//               accumulator into registers (packed BF16 after the FP32 bias
//               add), releases TMEM to the issuer, then stores its rows, so the
//               next tile's products overlap the global stores.
// Every wait is bounded; a timeout records a status bit and the CTA returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "host_common.h"
#include "sm100_ptx.cuh"
#include "tmem_io.cuh"

namespace erd {
namespace lin {

// Loads 16 consecutive 32-bit TMEM columns of this thread's lane and waits for
// them in the same asm statement.
__device__ __forceinline__ void tmem_ld_wait_16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

constexpr int kBN = 256;  // output columns per tile (one N=256 product)
constexpr int kRowBytes = 128;  // K bytes per stage and row: one 128-byte swizzle atom
// K elements per stage: 64 BF16 or 128 E4M3 (four K=16 or K=32 products either way).
template <bool kFp8>
constexpr int kBK = kFp8 ? 128 : 64;
constexpr int kBBytes = kBN * kRowBytes;  // 32 KB
constexpr int kEpilogueWarps = 8;
constexpr int kThreads = 32 * (2 + kEpilogueWarps);

// Tile geometry of the two instantiations: 256 output rows (two M=128
// accumulators filling TMEM, 3 stages) or 128 rows (one accumulator, two TMEM
// buffers so the epilogue of a tile overlaps the next tile's products, 4
// stages) for problems whose 256-row tiles would leave SMs idle.
template <int BM>
struct Tile {
  static constexpr int kAccs = BM / 128;     // M=128 accumulators per tile
  static constexpr int kBufs = 2 / kAccs;    // TMEM tile buffers
  static constexpr int kStages = BM == 128 ? 4 : 3;
  static constexpr int kABytes = BM * kRowBytes;
  static constexpr int kSmemA = 0;
  static constexpr int kSmemB = kSmemA + kStages * kABytes;
  static constexpr int kSmemBar = kSmemB + kStages * kBBytes;
  // Per epilogue warp, a 32-row x 64-column staging block (4 KB) for the
  // scattered columns, so that their stores leave as 128-byte row pieces.
  static constexpr int kSmemStage = kSmemBar + 1024;
  static constexpr int kStageBytes = 32 * 64 * 2;
  static constexpr int kSmemLaunchBytes = kSmemStage + 8 * kStageBytes + 1024;  // + base alignment
  static_assert(kSmemLaunchBytes <= 227 * 1024, "shared memory budget");
};

struct __align__(8) Barriers {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  int m, n, k;
  int tiles_m, tiles_n;
  int a_rows;  // rows of the x tile box (BM, or m when m < BM)
  const __nv_bfloat16* bias;  // [n] or null
  const float* col_scale;     // [n], E4M3 operands only: y = acc * col_scale + bias
  __nv_bfloat16* c;
  long long ldc;
  int* status;
  // Columns from scatter_col0 on (a multiple of 256) go to other buffers
  // instead of c: column j lands in scatter_base[g] with g = (j - scatter_col0)
  // >> scatter_group_shift, at (row / scatter_rows) * scatter_bs + (row %
  // scatter_rows) * scatter_ts + ((j - scatter_col0) & (group width - 1))
  // elements.  scatter_col0 == n: nothing is scattered.
  int scatter_col0;
  int scatter_group_shift;
  int scatter_rows;
  long long scatter_bs, scatter_ts;
  __nv_bfloat16* scatter_base[16];
};

template <int BM, bool kFp8, bool kScatter>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const Params p) {
  using T = Tile<BM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + T::kSmemBar);
  const uint32_t sA = smem_u32(smem + T::kSmemA);
  const uint32_t sB = smem_u32(smem + T::kSmemB);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = p.tiles_m * p.tiles_n;
  const int ksteps = p.k / kBK<kFp8>;
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bars->acc_full[b]), 1);
      mbar_init(smem_u32(&bars->acc_empty[b]), 32 * kEpilogueWarps);
    }
    mbar_init(smem_u32(&bars->mma_drain), 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      const uint32_t tx = static_cast<uint32_t>(p.a_rows * kRowBytes + kBBytes);
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * BM;
        const int n0 = (tile % p.tiles_n) * kBN;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = static_cast<int>(it % T::kStages);
          const uint32_t ph = (it / T::kStages) & 1;
          if (!mbar_wait(smem_u32(&bars->empty[s]), ph ^ 1, abort, p.status,
                         kStatusTimeoutProducer))
            break;
          mbar_arrive_expect_tx(smem_u32(&bars->full[s]), tx);
          tma_load_2d(sA + s * T::kABytes, &tmap_a, smem_u32(&bars->full[s]), kk * kBK<kFp8>,
                      m0);
          tma_load_2d(sB + s * kBBytes, &tmap_b, smem_u32(&bars->full[s]), kk * kBK<kFp8>, n0);
        }
      }
      if (*abort) {
        // Let the loads this thread may have started land before exiting.
        for (int d = 0; d < T::kStages && it > 0; ++d) {
          --it;
          mbar_wait_drain(smem_u32(&bars->full[it % T::kStages]), (it / T::kStages) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc =
          kFp8 ? idesc_e4m3_f32(128, kBN) : idesc_bf16_f32(128, kBN, false, false);
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++tcount) {
        const uint32_t buf = tcount % T::kBufs;
        // The epilogue has drained this TMEM buffer's previous tile.
        if (!mbar_wait(smem_u32(&bars->acc_empty[buf]), ((tcount / T::kBufs) & 1) ^ 1, abort,
                       p.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * T::kAccs * kBN;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = static_cast<int>(it % T::kStages);
          const uint32_t ph = (it / T::kStages) & 1;
          if (!mbar_wait(smem_u32(&bars->full[s]), ph, abort, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = sA + s * T::kABytes, b = sB + s * kBBytes;
#pragma unroll
          for (int h = 0; h < T::kAccs; ++h) {
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              // 32 bytes of K per product: 16 BF16 or 32 E4M3 values
              const uint64_t da = sdesc_sw128(a + h * 128 * kRowBytes + k4 * 32, 16, 1024);
              const uint64_t db = sdesc_sw128(b + k4 * 32, 16, 1024);
              const uint32_t acc = (kk > 0 || k4 > 0) ? 1u : 0u;
              if (kFp8)
                mma_f8_ss(d + h * kBN, da, db, idesc, acc);
              else
                mma_bf16_ss(d + h * kBN, da, db, idesc, acc);
            }
          }
          mma_commit(smem_u32(&bars->empty[s]));
        }
        if (!ok) break;
        mma_commit(smem_u32(&bars->acc_full[buf]));
      }
      mma_commit(smem_u32(&bars->mma_drain));
      mbar_wait_drain(smem_u32(&bars->mma_drain), 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp drains 32 rows (its TMEM lane quarter) of one accumulator:
    // all 256 columns with two accumulators, one 128-column half with one.
    constexpr int kCols = T::kAccs * 128;
    const int e = warp - 2;
    const int quad = warp & 3;
    const int h = T::kAccs == 2 ? (e >> 2) : 0;
    const int col0 = T::kAccs == 2 ? 0 : (e >> 2) * 128;
    const int row_in_tile = h * 128 + quad * 32 + lane;
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tcount) {
      const uint32_t buf = tcount % T::kBufs;
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->acc_full[buf]),
                                             (tcount / T::kBufs) & 1, abort, p.status,
                                             kStatusTimeoutEpilogue)))
        break;
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) +
                             (buf * T::kAccs + h) * kBN + col0;
      const int m0 = (tile / p.tiles_n) * BM;
      const int n0 = (tile % p.tiles_n) * kBN + col0;
      uint32_t out[kCols / 2];
#pragma unroll
      for (int c = 0; c < kCols / 16; ++c) {
        uint32_t r[16];
        tmem_ld_wait_16(taddr + c * 16, r);
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          uint4 w = make_uint4(0u, 0u, 0u, 0u);
          if (p.bias != nullptr)
            w = __ldg(reinterpret_cast<const uint4*>(p.bias + n0 + c * 16 + v * 8));
          const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
          float a[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) a[i] = __uint_as_float(r[8 * v + i]);
          if (kFp8) {
            const float4* cs = reinterpret_cast<const float4*>(p.col_scale + n0 + c * 16 + v * 8);
            const float4 c0 = __ldg(cs), c1 = __ldg(cs + 1);
            a[0] *= c0.x; a[1] *= c0.y; a[2] *= c0.z; a[3] *= c0.w;
            a[4] *= c1.x; a[5] *= c1.y; a[6] *= c1.z; a[7] *= c1.w;
          }
#pragma unroll
          for (int i = 0; i < 4; ++i)
            out[c * 8 + v * 4 + i] = pack_bf16x2(a[2 * i] + __uint_as_float(wv[i] << 16),
                                                 a[2 * i + 1] + __uint_as_float(wv[i] & 0xffff0000u));
        }
      }
      // The TMEM buffer is free for a later tile once every warp has read it.
      tc_fence_before();
      mbar_arrive(smem_u32(&bars->acc_empty[buf]));
      const int row = m0 + row_in_tile;
      if (!kScatter || n0 < p.scatter_col0) {
        if (row < p.m) {
          uint4* dst =
              reinterpret_cast<uint4*>(p.c + static_cast<long long>(row) * p.ldc + n0);
#pragma unroll
          for (int v = 0; v < kCols / 8; ++v)
            dst[v] = make_uint4(out[4 * v], out[4 * v + 1], out[4 * v + 2], out[4 * v + 3]);
        }
      } else {
        // Scattered columns (e.g. V straight into the peers' receive buffers,
        // over NVLink): 64 columns at a time go through this warp's staging
        // block, so that each store instruction writes four 128-byte row
        // pieces instead of 32 separate 16-byte ones.
        const int b = row / p.scatter_rows;
        const long long my_off =
            b * p.scatter_bs + static_cast<long long>(row - b * p.scatter_rows) * p.scatter_ts;
        const int mask = (1 << p.scatter_group_shift) - 1;
        uint8_t* stage = smem + T::kSmemStage + e * T::kStageBytes;
        const int sub = lane >> 3, chunk = lane & 7;  // row within a group of 4, 16-byte chunk
#pragma unroll
        for (int piece = 0; piece < kCols / 64; ++piece) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int v = piece * 8 + c;
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) * 16)) =
                make_uint4(out[4 * v], out[4 * v + 1], out[4 * v + 2], out[4 * v + 3]);
          }
          __syncwarp();
          const int j = n0 + piece * 64 + chunk * 8 - p.scatter_col0;
          __nv_bfloat16* base = p.scatter_base[j >> p.scatter_group_shift] + (j & mask);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int rr = 4 * q + sub;  // staged row (the lane that drained it)
            const long long off = __shfl_sync(0xffffffffu, my_off, rr);
            const bool valid = __shfl_sync(0xffffffffu, row < p.m ? 1 : 0, rr) != 0;
            const uint4 val =
                *reinterpret_cast<const uint4*>(stage + rr * 128 + ((chunk ^ (rr & 7)) * 16));
            if (valid) *reinterpret_cast<uint4*>(base + off) = val;
          }
          __syncwarp();
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace lin
}  // namespace erd

using namespace erd;

namespace {

// Shared host path of the BF16 and E4M3 entry points: argument checks, tensor
// maps, tile height and launch.
template <int BM, bool kFp8, bool kScatter>
cudaError_t launch_linear(unsigned grid, cudaStream_t st, const CUtensorMap& ta,
                          const CUtensorMap& tb, const lin::Params& p) {
  using namespace erd::lin;
  cudaError_t e = cudaFuncSetAttribute(linear_kernel<BM, kFp8, kScatter>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Tile<BM>::kSmemLaunchBytes);
  if (e != cudaSuccess) return e;
  linear_kernel<BM, kFp8, kScatter><<<grid, kThreads, Tile<BM>::kSmemLaunchBytes, st>>>(ta, tb, p);
  return cudaGetLastError();
}

struct Scatter {
  int col0, group_shift, rows;
  int64_t bs, ts;
  void* const* bases;
  int nbases;
};

template <bool kFp8>
int linear_launch(const void* x, int64_t ldx, const void* weight, int64_t ldw,
                  const float* col_scale, const void* bias, void* y, int64_t ldy, int m, int n,
                  int k, int* status, void* stream, const Scatter* scatter = nullptr) {
  using namespace erd::lin;
  constexpr int elem = kFp8 ? 1 : 2;  // bytes per operand element
  if (x == nullptr || weight == nullptr || y == nullptr || (kFp8 && col_scale == nullptr))
    return kErrNullPointer;
  if (m <= 0 || n <= 0 || k <= 0 || n % kBN != 0 || k % kBK<kFp8> != 0) return kErrBadShape;
  if (ldx < k || ldw < k || ldy < n) return kErrBadShape;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(y) ||
      (bias != nullptr && !aligned16(bias)) || (col_scale != nullptr && !aligned16(col_scale)) ||
      (ldx * elem) % 16 != 0 || (ldw * elem) % 16 != 0 || (ldy & 7) != 0)
    return kErrMisaligned;
  if (int rc = check_device_sm100()) return rc;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  // Tile height: 256 rows unless 128-row tiles finish sooner on this many SMs.
  // Measured on B200 at K = 2048 (BF16): a wave of 128-row tiles takes 0.527
  // of a wave of 256-row ones, and a launch pays about 0.3 of a 256-row tile
  // in pipeline fill and drain.
  const long long tiles_n = n / kBN;
  const long long t256 = (m + 255) / 256 * tiles_n, t128 = (m + 127) / 128 * tiles_n;
  const long long w256 = (t256 + sms - 1) / sms, w128 = (t128 + sms - 1) / sms;
  const int bm = (w128 * 527 < w256 * 1000 + 300) ? 128 : 256;
  if (t128 > (1LL << 30)) return kErrTooLarge;

  const CUtensorMapDataType dtype =
      kFp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta, tb;
  const int a_rows = m < bm ? m : bm;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldx) * elem};
    const uint32_t box[2] = {kBK<kFp8>, static_cast<uint32_t>(a_rows)};
    if (encode_tensor_map(&ta, dtype, 2, const_cast<void*>(x), dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return kErrTensorMap;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldw) * elem};
    const uint32_t box[2] = {kBK<kFp8>, kBN};
    if (encode_tensor_map(&tb, dtype, 2, const_cast<void*>(weight), dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return kErrTensorMap;
  }
  Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_m = (m + bm - 1) / bm;
  p.tiles_n = static_cast<int>(tiles_n);
  p.a_rows = a_rows;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.col_scale = col_scale;
  p.c = static_cast<__nv_bfloat16*>(y);
  p.ldc = ldy;
  p.status = status;
  p.scatter_col0 = n;
  p.scatter_group_shift = 0;
  p.scatter_rows = 1;
  p.scatter_bs = p.scatter_ts = 0;
  for (int g = 0; g < 16; ++g) p.scatter_base[g] = nullptr;
  if (scatter != nullptr) {
    p.scatter_col0 = scatter->col0;
    p.scatter_group_shift = scatter->group_shift;
    p.scatter_rows = scatter->rows;
    p.scatter_bs = scatter->bs;
    p.scatter_ts = scatter->ts;
    for (int g = 0; g < scatter->nbases; ++g)
      p.scatter_base[g] = static_cast<__nv_bfloat16*>(scatter->bases[g]);
  }
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  const unsigned grid = static_cast<unsigned>(tiles < sms ? tiles : sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (scatter != nullptr) {
    if constexpr (kFp8) {
      return kErrBadShape;  // the scattered epilogue serves the BF16 product only
    } else {
      e = bm == 128 ? launch_linear<128, false, true>(grid, st, ta, tb, p)
                    : launch_linear<256, false, true>(grid, st, ta, tb, p);
    }
  } else {
    e = bm == 128 ? launch_linear<128, kFp8, false>(grid, st, ta, tb, p)
                  : launch_linear<256, kFp8, false>(grid, st, ta, tb, p);
  }
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" int erd_linear_bf16(const void* x, int64_t ldx, const void* weight, int64_t ldw,
                               const void* bias, void* y, int64_t ldy, int m, int n, int k,
                               int* status, void* stream) {
  return linear_launch<false>(x, ldx, weight, ldw, nullptr, bias, y, ldy, m, n, k, status,
                              stream);
}

extern "C" int erd_linear_bf16_scatter(const void* x, int64_t ldx, const void* weight,
                                       int64_t ldw, const void* bias, void* y, int64_t ldy, int m,
                                       int n, int k, int scatter_col0, void* const* dest_bases,
                                       int ndest, int group_cols, int rows_per_batch,
                                       int64_t dest_batch_stride, int64_t dest_token_stride,
                                       int* status, void* stream) {
  if (dest_bases == nullptr) return kErrNullPointer;
  if (ndest <= 0 || ndest > 16 || group_cols < 128 || (group_cols & (group_cols - 1)) != 0 ||
      scatter_col0 < 0 || scatter_col0 % erd::lin::kBN != 0 ||
      static_cast<long long>(ndest) * group_cols != static_cast<long long>(n) - scatter_col0 ||
      rows_per_batch <= 0 || m % rows_per_batch != 0 || dest_batch_stride < 0 ||
      dest_token_stride < 0)
    return kErrBadShape;
  if (((dest_batch_stride | dest_token_stride) & 7) != 0) return kErrMisaligned;
  for (int g = 0; g < ndest; ++g) {
    if (dest_bases[g] == nullptr) return kErrNullPointer;
    if (!aligned16(dest_bases[g])) return kErrMisaligned;
  }
  int shift = 0;
  while ((1 << shift) < group_cols) ++shift;
  const Scatter sc{scatter_col0, shift, rows_per_batch, dest_batch_stride, dest_token_stride,
                   dest_bases, ndest};
  // y is only written below scatter_col0; with nothing local it still passes
  // the common checks (and is never dereferenced).
  return linear_launch<false>(x, ldx, weight, ldw, nullptr, bias, y, ldy, m, n, k, status,
                              stream, &sc);
}

extern "C" int erd_linear_fp8(const void* x, int64_t ldx, const void* weight, int64_t ldw,
                              const float* col_scale, const void* bias, void* y, int64_t ldy,
                              int m, int n, int k, int* status, void* stream) {
  return linear_launch<true>(x, ldx, weight, ldw, col_scale, bias, y, ldy, m, n, k, status,
                             stream);
}
