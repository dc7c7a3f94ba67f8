// Fused QK RMSNorm-across-heads + LTX 3D RoPE prologue, plus the per-axis
// RoPE table builder.
//
// One warp per token.  Lane i owns the eight 16-byte chunks
// c = 256 * it + 8 * i (it = 0..7) of the 2048-wide Q and K rows, so every
// warp-wide load / store instruction moves 512 contiguous bytes.  Rounding
// follows the unfused reference exactly: fp32 sum of squares, r = rsqrt(mean
// + eps), y = bf16(x * r), z = bf16(y * w), out = bf16(z * cos + rot(z) * sin)
// with separately rounded products (no FMA contraction), as in
// models/dits/eraserdit_attention.py:68-79 and
// layers/operator_fusion/triton/rmsnorm_native.py:25-43.  Only the order of
// the fp32 sum of squares differs from torch's reduction.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/eraserdit_b200.h"
#include "host_common.h"

namespace erd {

constexpr int kHidden = 2048;
constexpr int kHeadDimP = 64;
constexpr int kChunksPerLane = kHidden / 256;  // 8 chunks of 8 elements
constexpr int kTokensPerBlock = 4;
// Blocks per SM the register budget is sized for: 8 x 4 warps at <= 64
// registers.  Measured at configuration 1 (2 x 32640 tokens): 3 blocks
// (rows held in registers) 0.32 ms, 5 blocks 0.27 ms, 8 blocks 0.25 ms,
// 10 blocks (spills) 0.23 ms vs 0.217 ms for 8 with the table pointers below.
constexpr int kPrologueBlocksPerSm = 8;

struct PrologueParams {
  const __nv_bfloat16* q_in;
  const __nv_bfloat16* k_in;
  const __nv_bfloat16* v_in;
  long long in_ts, in_bs;
  int batch, tokens;
  const __nv_bfloat16* wq;
  const __nv_bfloat16* wk;
  float eps;
  const float* cos_tab;
  const float* sin_tab;
  long long tab_ts, tab_bs;
  const float2* axis_tab;
  int nfreq, grid_f, grid_h, grid_w, token_offset;
  const int* grid_index;  // optional: grid position of each token (tokens laid out in another order)
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  long long out_ts, out_bs, out_hs, out_ds;
  int heads_per_dest;
  // Peer mode: head group g goes to dest_base[g] (another rank's receive
  // buffer), Q at +0, K at +k_rel, V at +v_rel elements.
  __nv_bfloat16* dest_base[16];
  long long k_rel, v_rel;
  int peer;
};


__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Two values rounded to BF16 (nearest even) by one packed conversion.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void bf16_round2(float& a, float& b) {
  const uint32_t r = cvt_bf16x2(a, b);
  a = __uint_as_float(r << 16);
  b = __uint_as_float(r & 0xFFFF0000u);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(cvt_bf16x2(f[0], f[1]), cvt_bf16x2(f[2], f[3]), cvt_bf16x2(f[4], f[5]),
                    cvt_bf16x2(f[6], f[7]));
}

// y = bf16(x * r), then z = bf16(y * w) when an affine weight is present.
__device__ __forceinline__ void norm8(float (&x)[8], float r, const __nv_bfloat16* w, int c0) {
  float wf[8];
  if (w != nullptr) {
    unpack8(__ldg(reinterpret_cast<const uint4*>(w + c0)), wf);
  }
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    float y0 = __fmul_rn(x[e], r), y1 = __fmul_rn(x[e + 1], r);
    bf16_round2(y0, y1);
    if (w != nullptr) {
      y0 = __fmul_rn(y0, wf[e]);
      y1 = __fmul_rn(y1, wf[e + 1]);
      bf16_round2(y0, y1);
    }
    x[e] = y0;
    x[e + 1] = y1;
  }
}

// out[2i] = z[2i] cos[2i] - z[2i+1] sin[2i]; out[2i+1] = z[2i+1] cos[2i+1] + z[2i] sin[2i+1]
__device__ __forceinline__ void rope8(float (&z)[8], const float (&cs)[8], const float (&sn)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = z[2 * i], b = z[2 * i + 1];
    z[2 * i] = __fadd_rn(__fmul_rn(a, cs[2 * i]), __fmul_rn(-b, sn[2 * i]));
    z[2 * i + 1] = __fadd_rn(__fmul_rn(b, cs[2 * i + 1]), __fmul_rn(a, sn[2 * i + 1]));
  }
}

template <int kRopeMode, bool kHasK>
__global__ void __launch_bounds__(kTokensPerBlock * 32, kPrologueBlocksPerSm)
    qk_norm_rope_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const long long g = static_cast<long long>(blockIdx.x) * kTokensPerBlock + (threadIdx.x >> 5);
  if (g >= static_cast<long long>(p.batch) * p.tokens) return;
  const int b = static_cast<int>(g / p.tokens);
  const int t = static_cast<int>(g - static_cast<long long>(b) * p.tokens);

  // V is only repacked: copy it first so that its registers are free again
  // before Q and K are loaded.
  if (p.v_in != nullptr && p.v_out != nullptr) {
    const __nv_bfloat16* vrow = p.v_in + b * p.in_bs + t * p.in_ts;
    uint4 vv[kChunksPerLane];
#pragma unroll
    for (int it = 0; it < kChunksPerLane; ++it)
      vv[it] = *reinterpret_cast<const uint4*>(vrow + it * 256 + lane * 8);
#pragma unroll
    for (int it = 0; it < kChunksPerLane; ++it) {
      const int c0 = it * 256 + lane * 8;
      const int head = c0 / kHeadDimP;
      const int dest = head / p.heads_per_dest;
      const int hl = head - dest * p.heads_per_dest;
      const long long off = b * p.out_bs + t * p.out_ts + hl * p.out_hs + (c0 - head * kHeadDimP);
      __nv_bfloat16* dst = p.peer ? p.dest_base[dest] + p.v_rel : p.v_out + dest * p.out_ds;
      *reinterpret_cast<uint4*>(dst + off) = vv[it];
    }
  }

  const __nv_bfloat16* qrow = p.q_in + b * p.in_bs + t * p.in_ts;
  const __nv_bfloat16* krow = p.k_in + b * p.in_bs + t * p.in_ts;

  // fp32 sum of squares over the full 2048-wide rows (squares of BF16 values
  // are exact in fp32).  Four partial sums per lane keep the dependent-add
  // chains short.  The rows are not kept in registers: the second pass reads
  // them again (from L1), which leaves room for more tokens in flight per SM.
  float sq4[4] = {0.f, 0.f, 0.f, 0.f}, sk4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int it = 0; it < kChunksPerLane; ++it) {
    const int c0 = it * 256 + lane * 8;
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(qrow + c0), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) sq4[e & 3] = __fmaf_rn(f[e], f[e], sq4[e & 3]);
    if (kHasK) {
      unpack8(*reinterpret_cast<const uint4*>(krow + c0), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) sk4[e & 3] = __fmaf_rn(f[e], f[e], sk4[e & 3]);
    }
  }
  float sq = (sq4[0] + sq4[1]) + (sq4[2] + sq4[3]);
  float sk = (sk4[0] + sk4[1]) + (sk4[2] + sk4[3]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, off);
    sk += __shfl_xor_sync(0xffffffffu, sk, off);
  }
  // 1 / sqrt with IEEE rounding of both steps, as torch's CPU rsqrt computes it.
  const float rq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq * (1.0f / kHidden), p.eps)));
  const float rk = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sk * (1.0f / kHidden), p.eps)));

  // RoPE from the per-axis table.  Channel pair (c, c+1), c even: c < 2 is
  // the identity; otherwise pair index pr = (c - 2) / 2 uses frequency pr / 3
  // on axis pr % 3 (eraserdit_transformer.py:202-212), i.e. table entry
  // row[axis] + pr / 3 with row[axis] the start of this token's coordinate
  // on that axis.  The pairs of lane l in chunk it are pr = pr0 + d with
  // pr0 = 4 l - 1 and d = 128 it + i (i = 0..3, known at compile time):
  // with d = 3 dq + dm, the entry is ptr[dm][dq], ptr[dm] = row[(a0 + dm) % 3]
  // + k0 + (a0 + dm) / 3, where k0 = floor(pr0 / 3) and a0 = pr0 - 3 k0.
  const float2* rope_ptr[3] = {nullptr, nullptr, nullptr};
  if (kRopeMode == 2) {
    const int gpos = p.grid_index != nullptr ? __ldg(p.grid_index + p.token_offset + t)
                                             : p.token_offset + t;
    const int hw = p.grid_h * p.grid_w;
    const int pos_f = gpos / hw;
    const int rem = gpos - pos_f * hw;
    const int pos_h = rem / p.grid_w;
    const int pos_w = rem - pos_h * p.grid_w;
    const int row[3] = {pos_f * p.nfreq, (p.grid_f + pos_h) * p.nfreq,
                        (p.grid_f + p.grid_h + pos_w) * p.nfreq};
    const int pr0 = 4 * lane - 1;
    const int k0 = lane == 0 ? -1 : pr0 / 3;
    const int a0 = pr0 - 3 * k0;
#pragma unroll
    for (int dm = 0; dm < 3; ++dm) {
      const int a = a0 + dm;
      const int axis = a >= 3 ? a - 3 : a;
      const int r = axis == 0 ? row[0] : (axis == 1 ? row[1] : row[2]);
      rope_ptr[dm] = p.axis_tab + r + k0 + (a >= 3 ? 1 : 0);
    }
  }

#pragma unroll
  for (int it = 0; it < kChunksPerLane; ++it) {
    const int c0 = it * 256 + lane * 8;
    float q[8], k[8];
    unpack8(*reinterpret_cast<const uint4*>(qrow + c0), q);
    norm8(q, rq, p.wq, c0);
    if (kHasK) {
      unpack8(*reinterpret_cast<const uint4*>(krow + c0), k);
      norm8(k, rk, p.wk, c0);
    }
    if (kRopeMode != 0) {
      float cs[8], sn[8];
      if (kRopeMode == 1) {
        const float* cb = p.cos_tab + b * p.tab_bs + t * p.tab_ts + c0;
        const float* sb = p.sin_tab + b * p.tab_bs + t * p.tab_ts + c0;
        const float4 c_lo = __ldg(reinterpret_cast<const float4*>(cb));
        const float4 c_hi = __ldg(reinterpret_cast<const float4*>(cb + 4));
        const float4 s_lo = __ldg(reinterpret_cast<const float4*>(sb));
        const float4 s_hi = __ldg(reinterpret_cast<const float4*>(sb + 4));
        cs[0] = c_lo.x; cs[1] = c_lo.y; cs[2] = c_lo.z; cs[3] = c_lo.w;
        cs[4] = c_hi.x; cs[5] = c_hi.y; cs[6] = c_hi.z; cs[7] = c_hi.w;
        sn[0] = s_lo.x; sn[1] = s_lo.y; sn[2] = s_lo.z; sn[3] = s_lo.w;
        sn[4] = s_hi.x; sn[5] = s_hi.y; sn[6] = s_hi.z; sn[7] = s_hi.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = it * 128 + i;
          // pr = -1 (lane 0, first pair): the two leading channels are unrotated.
          const bool identity = it == 0 && i == 0 && lane == 0;
          const float2 e = identity ? make_float2(1.f, 0.f) : __ldg(rope_ptr[d % 3] + d / 3);
          cs[2 * i] = e.x;
          cs[2 * i + 1] = e.x;
          sn[2 * i] = e.y;
          sn[2 * i + 1] = e.y;
        }
      }
      rope8(q, cs, sn);
      rope8(k, cs, sn);
    }
    const int head = c0 / kHeadDimP;
    const int d0 = c0 - head * kHeadDimP;
    const int dest = head / p.heads_per_dest;
    const int hl = head - dest * p.heads_per_dest;
    const long long off = b * p.out_bs + t * p.out_ts + hl * p.out_hs + d0;
    if (p.peer) {
      __nv_bfloat16* base = p.dest_base[dest];
      *reinterpret_cast<uint4*>(base + off) = pack8(q);
      if (kHasK) *reinterpret_cast<uint4*>(base + p.k_rel + off) = pack8(k);
    } else {
      *reinterpret_cast<uint4*>(p.q_out + dest * p.out_ds + off) = pack8(q);
      if (kHasK) *reinterpret_cast<uint4*>(p.k_out + dest * p.out_ds + off) = pack8(k);
    }
  }
}

// One thread per (axis, coordinate, frequency) entry.
__global__ void rope_axis_table_kernel(const float* __restrict__ freqs, int nfreq, int frames,
                                       int height, int width, int use_scale, float scale_f,
                                       float scale_h, float scale_w, float patch_t, float patch_s,
                                       float base_f, float base_h, float base_w,
                                       float2* __restrict__ table) {
  const int total = (frames + height + width) * nfreq;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int kf = idx % nfreq;
  const int i_all = idx / nfreq;
  float coord;
  if (i_all < frames) {
    coord = static_cast<float>(i_all);
    if (use_scale) coord = __fdiv_rn(__fmul_rn(__fmul_rn(coord, scale_f), patch_t), base_f);
  } else if (i_all < frames + height) {
    coord = static_cast<float>(i_all - frames);
    if (use_scale) coord = __fdiv_rn(__fmul_rn(__fmul_rn(coord, scale_h), patch_s), base_h);
  } else {
    coord = static_cast<float>(i_all - frames - height);
    if (use_scale) coord = __fdiv_rn(__fmul_rn(__fmul_rn(coord, scale_w), patch_s), base_w);
  }
  const float angle = __fmul_rn(freqs[kf], __fadd_rn(__fmul_rn(coord, 2.0f), -1.0f));
  float s, c;
  sincosf(angle, &s, &c);
  table[idx] = make_float2(c, s);
}

}  // namespace erd

using namespace erd;

extern "C" int erd_rope_axis_table(const float* freqs, int nfreq, int frames, int height, int width,
                                   int use_scale, float scale_f, float scale_h, float scale_w,
                                   float patch_t, float patch_s, float base_f, float base_h,
                                   float base_w, float* table, void* stream) {
  if (freqs == nullptr || table == nullptr) return kErrNullPointer;
  if (nfreq <= 0 || frames <= 0 || height <= 0 || width <= 0) return kErrBadShape;
  if (int rc = check_device_sm100()) return rc;
  const int total = (frames + height + width) * nfreq;
  rope_axis_table_kernel<<<(total + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      freqs, nfreq, frames, height, width, use_scale, scale_f, scale_h, scale_w, patch_t, patch_s,
      base_f, base_h, base_w, reinterpret_cast<float2*>(table));
  return static_cast<int>(cudaGetLastError());
}

namespace {

struct PeerOut {
  void* const* dest_bases;
  int ndest;
  int64_t k_rel, v_rel;
};

int qk_norm_rope_impl(const void* q_in, const void* k_in, const void* v_in,
                      int64_t in_token_stride, int64_t in_batch_stride, int batch, int tokens,
                      int hidden, const void* q_weight, const void* k_weight, float eps,
                      int rope_mode, const float* cos_tab, const float* sin_tab,
                      int64_t tab_token_stride, int64_t tab_batch_stride,
                      const float* axis_table, int nfreq, int frames, int height, int width,
                      int token_offset, const int32_t* grid_index, void* q_out, void* k_out,
                      void* v_out, int64_t out_token_stride, int64_t out_batch_stride,
                      int64_t out_head_stride, int heads_per_dest, int64_t out_dest_stride,
                      const PeerOut* peer, void* stream) {
  // Q alone (k_in and k_out NULL): the cross-attention query norm, no RoPE, no V.
  const bool q_only = k_in == nullptr && k_out == nullptr;
  if (q_in == nullptr || q_out == nullptr || (!q_only && (k_in == nullptr || k_out == nullptr)))
    return kErrNullPointer;
  if (q_only && (rope_mode != 0 || v_in != nullptr || peer != nullptr)) return kErrBadShape;
  if (hidden != kHidden || batch < 0 || tokens < 0 || heads_per_dest <= 0 ||
      (kHidden / kHeadDimP) % heads_per_dest != 0)
    return kErrBadShape;
  if (rope_mode < 0 || rope_mode > 2) return kErrBadShape;
  if (grid_index != nullptr && rope_mode != 2) return kErrBadShape;
  if (rope_mode == 1 && (cos_tab == nullptr || sin_tab == nullptr)) return kErrNullPointer;
  if (rope_mode == 2) {
    if (axis_table == nullptr) return kErrNullPointer;
    if (nfreq != kHidden / 6 || frames <= 0 || height <= 0 || width <= 0 || token_offset < 0 ||
        static_cast<long long>(token_offset) + tokens >
            static_cast<long long>(frames) * height * width)
      return kErrBadShape;
  }
  const void* ptrs[] = {q_in, k_in, q_out, k_out, q_weight, k_weight, v_in, v_out};
  for (const void* ptr : ptrs)
    if (ptr != nullptr && !aligned16(ptr)) return kErrMisaligned;
  if ((in_token_stride | in_batch_stride | out_token_stride | out_batch_stride | out_head_stride |
       out_dest_stride) & 7)
    return kErrMisaligned;
  if (rope_mode == 1 && (!aligned16(cos_tab) || !aligned16(sin_tab) ||
                         ((tab_token_stride | tab_batch_stride) & 3)))
    return kErrMisaligned;
  if (int rc = check_device_sm100()) return rc;
  if (batch == 0 || tokens == 0) return kErrOk;

  PrologueParams p;
  p.q_in = static_cast<const __nv_bfloat16*>(q_in);
  p.k_in = static_cast<const __nv_bfloat16*>(k_in);
  p.v_in = static_cast<const __nv_bfloat16*>(v_in);
  p.in_ts = in_token_stride;
  p.in_bs = in_batch_stride;
  p.batch = batch;
  p.tokens = tokens;
  p.wq = static_cast<const __nv_bfloat16*>(q_weight);
  p.wk = static_cast<const __nv_bfloat16*>(k_weight);
  p.eps = eps;
  p.cos_tab = cos_tab;
  p.sin_tab = sin_tab;
  p.tab_ts = tab_token_stride;
  p.tab_bs = tab_batch_stride;
  p.axis_tab = reinterpret_cast<const float2*>(axis_table);
  p.nfreq = nfreq;
  p.grid_f = frames;
  p.grid_h = height;
  p.grid_w = width;
  p.token_offset = token_offset;
  p.grid_index = grid_index;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.v_out = static_cast<__nv_bfloat16*>(v_out);
  p.out_ts = out_token_stride;
  p.out_bs = out_batch_stride;
  p.out_hs = out_head_stride;
  p.out_ds = out_dest_stride;
  p.heads_per_dest = heads_per_dest;
  p.peer = 0;
  p.k_rel = p.v_rel = 0;
  for (int g = 0; g < 16; ++g) p.dest_base[g] = nullptr;
  if (peer != nullptr) {
    if (peer->dest_bases == nullptr) return kErrNullPointer;
    if (peer->ndest != (kHidden / kHeadDimP) / heads_per_dest || peer->ndest > 16)
      return kErrBadShape;
    if ((peer->k_rel | peer->v_rel) & 7) return kErrMisaligned;
    for (int g = 0; g < peer->ndest; ++g) {
      p.dest_base[g] = static_cast<__nv_bfloat16*>(peer->dest_bases[g]);
      if (p.dest_base[g] == nullptr) return kErrNullPointer;
      if (!aligned16(p.dest_base[g])) return kErrMisaligned;
    }
    p.k_rel = peer->k_rel;
    p.v_rel = peer->v_rel;
    p.peer = 1;
  }

  const long long rows = static_cast<long long>(batch) * tokens;
  const unsigned grid = static_cast<unsigned>((rows + kTokensPerBlock - 1) / kTokensPerBlock);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (q_only) {
    qk_norm_rope_kernel<0, false><<<grid, kTokensPerBlock * 32, 0, s>>>(p);
    return static_cast<int>(cudaGetLastError());
  }
  switch (rope_mode) {
    case 0: qk_norm_rope_kernel<0, true><<<grid, kTokensPerBlock * 32, 0, s>>>(p); break;
    case 1: qk_norm_rope_kernel<1, true><<<grid, kTokensPerBlock * 32, 0, s>>>(p); break;
    default: qk_norm_rope_kernel<2, true><<<grid, kTokensPerBlock * 32, 0, s>>>(p); break;
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" int erd_qk_norm_rope(const void* q_in, const void* k_in, const void* v_in,
                                int64_t in_token_stride, int64_t in_batch_stride, int batch,
                                int tokens, int hidden, const void* q_weight, const void* k_weight,
                                float eps, int rope_mode, const float* cos_tab,
                                const float* sin_tab, int64_t tab_token_stride,
                                int64_t tab_batch_stride, const float* axis_table, int nfreq,
                                int frames, int height, int width, int token_offset,
                                const int32_t* grid_index, void* q_out,
                                void* k_out, void* v_out, int64_t out_token_stride,
                                int64_t out_batch_stride, int64_t out_head_stride,
                                int heads_per_dest, int64_t out_dest_stride, void* stream) {
  return qk_norm_rope_impl(q_in, k_in, v_in, in_token_stride, in_batch_stride, batch, tokens,
                           hidden, q_weight, k_weight, eps, rope_mode, cos_tab, sin_tab,
                           tab_token_stride, tab_batch_stride, axis_table, nfreq, frames, height,
                           width, token_offset, grid_index, q_out, k_out, v_out, out_token_stride,
                           out_batch_stride, out_head_stride, heads_per_dest, out_dest_stride,
                           nullptr, stream);
}

extern "C" int erd_qk_norm_rope_peer(const void* q_in, const void* k_in, const void* v_in,
                                     int64_t in_token_stride, int64_t in_batch_stride, int batch,
                                     int tokens, int hidden, const void* q_weight,
                                     const void* k_weight, float eps, int rope_mode,
                                     const float* cos_tab, const float* sin_tab,
                                     int64_t tab_token_stride, int64_t tab_batch_stride,
                                     const float* axis_table, int nfreq, int frames, int height,
                                     int width, int token_offset, const int32_t* grid_index,
                                     void* const* dest_bases, int ndest, int64_t k_offset,
                                     int64_t v_offset, int64_t out_token_stride,
                                     int64_t out_batch_stride, int64_t out_head_stride,
                                     int heads_per_dest, void* stream) {
  if (dest_bases == nullptr || ndest <= 0) return kErrNullPointer;
  const PeerOut peer{dest_bases, ndest, k_offset, v_offset};
  // q_out / k_out only pass the null checks: every store goes through dest_bases.
  return qk_norm_rope_impl(q_in, k_in, v_in, in_token_stride, in_batch_stride, batch, tokens,
                           hidden, q_weight, k_weight, eps, rope_mode, cos_tab, sin_tab,
                           tab_token_stride, tab_batch_stride, axis_table, nfreq, frames, height,
                           width, token_offset, grid_index, dest_bases[0], dest_bases[0],
                           v_in != nullptr ? dest_bases[0] : nullptr, out_token_stride,
                           out_batch_stride, out_head_stride, heads_per_dest, 0, &peer, stream);
}
