// Token-batched kernels around the tensor-core GEMM (tc_gemm.cuh): embedding rows, decode
// attention for many (token, kv head) pairs, and per-row greedy argmax.  Each token carries its
// own sequence slot and position, so one launch serves batched decode (one token per sequence)
// and prefill (consecutive positions of one sequence; causality comes from each token reading
// the cache only up to its own position).
#pragma once

#include "decode_kernels.cuh"

namespace le {

// x[t] = dequantised row tok[t] of the tied lm_head (dequantize_embedding_row,
// src/llama_engine.cpp:182-220).
__global__ void k_embed_batch(QMat E, const int32_t* __restrict__ tok, float* __restrict__ x, int ldx) {
  const int t = blockIdx.x;
  const int token = tok[t];
  const int K = E.K, nb = K >> 7;
  float* out = x + (size_t)t * ldx;
  for (int k2 = threadIdx.x; k2 < K / 2; k2 += blockDim.x) {
    const int b = k2 >> 6;
    const size_t blk = (size_t)token * nb + b;
    const float st = bf16_bits_to_f32(E.step[blk]);
    const float mv = bf16_bits_to_f32(E.mn[blk]);
    const uint32_t byte = E.nib[(size_t)token * (K >> 1) + k2];
    out[2 * k2] = __fadd_rn(mv, __fmul_rn((float)(byte & 0xFu), st));
    out[2 * k2 + 1] = __fadd_rn(mv, __fmul_rn((float)(byte >> 4), st));
  }
}

// Attention of token t (position pos[t], sequence slot[t]) for the 4 q heads of kv head g
// (src/llama_engine.cpp:958-1021: kv_h = h / 4, s = (q . k) * 0.125, softmax over 0..pos,
// o = sum p v).  The token's own k / v are already in the cache (written by the QKV epilogue).
// One CTA of 4 warps per (t, g); warp w takes 32-position tiles w, w+4, ...: lane = position
// for the scores (its k row read whole), lane = dimension pair for p . v (v rows read
// coalesced); both loads of a tile are issued before either is used.  Softmax runs online per
// warp (running max and sum, rescaled per tile); the four warps' partial results are merged at
// the end.
__global__ void __launch_bounds__(128, 3)
    k_attn_batch(const float* __restrict__ q, int q_dim, const float* __restrict__ kc, const float* __restrict__ vc,
                 size_t slot_stride, int kv_dim, const int32_t* __restrict__ pos, const int32_t* __restrict__ slot,
                 float* __restrict__ out) {
  __shared__ float4 sq4[64];      // (q_h0[d], q_h1[d], q_h2[d], q_h3[d])
  __shared__ float4 sp[4][32];    // per warp: softmax numerators of the tile, 4 heads per position
  __shared__ float s_m[4][4], s_l[4][4];
  __shared__ float s_o[4][4][64];
  const int t = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = pos[t] + 1;
  const size_t base = (size_t)slot[t] * slot_stride + (size_t)g * LE_HEAD_DIM;
  const float* Kb = kc + base;
  const float* Vb = vc + base;
  if (threadIdx.x < 64) {
    const float* qh = q + (size_t)t * q_dim + (size_t)(4 * g) * LE_HEAD_DIM + threadIdx.x;
    sq4[threadIdx.x] = make_float4(qh[0], qh[64], qh[128], qh[192]);
  }
  __syncthreads();
  float m[4], l[4], o[4][2];
#pragma unroll
  for (int h = 0; h < 4; ++h) { m[h] = -INFINITY; l[h] = 0.0f; o[h][0] = 0.0f; o[h][1] = 0.0f; }
  for (int j = warp; j * 32 < P; j += 4) {
    const int p = j * 32 + lane;
    const int nv = min(32, P - j * 32);
    // the tile's k row (this lane's position) and v rows (this lane's two dimensions of all 32
    // positions) are requested together: one memory round trip per tile
    float4 kv[16];
    float2 vv[32];
    const float* kr = Kb + (size_t)min(p, P - 1) * kv_dim;
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) kv[d4] = *reinterpret_cast<const float4*>(kr + 4 * d4);
    const float* vr = Vb + (size_t)(j * 32) * kv_dim + 2 * lane;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      vv[i] = i < nv ? *reinterpret_cast<const float2*>(vr + (size_t)i * kv_dim) : make_float2(0.0f, 0.0f);
    float s[4];
    {
      float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int d4 = 0; d4 < 16; ++d4) {
        const float ke[4] = {kv[d4].x, kv[d4].y, kv[d4].z, kv[d4].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 qq = sq4[4 * d4 + e];
          dot[0] = fmaf(qq.x, ke[e], dot[0]);
          dot[1] = fmaf(qq.y, ke[e], dot[1]);
          dot[2] = fmaf(qq.z, ke[e], dot[2]);
          dot[3] = fmaf(qq.w, ke[e], dot[3]);
        }
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) s[h] = p < P ? dot[h] * 0.125f : -INFINITY;
    }
    float pe[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float mn = fmaxf(m[h], warp_max(s[h]));  // finite: the tile holds a valid position
      const float alpha = expf(m[h] - mn);
      pe[h] = expf(s[h] - mn);
      l[h] = l[h] * alpha + warp_sum(pe[h]);
      o[h][0] *= alpha;
      o[h][1] *= alpha;
      m[h] = mn;
    }
    sp[warp][lane] = make_float4(pe[0], pe[1], pe[2], pe[3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) {  // positions past the tile's end have p = 0 and v = 0
      const float4 pp = sp[warp][i];
      o[0][0] = fmaf(pp.x, vv[i].x, o[0][0]); o[0][1] = fmaf(pp.x, vv[i].y, o[0][1]);
      o[1][0] = fmaf(pp.y, vv[i].x, o[1][0]); o[1][1] = fmaf(pp.y, vv[i].y, o[1][1]);
      o[2][0] = fmaf(pp.z, vv[i].x, o[2][0]); o[2][1] = fmaf(pp.z, vv[i].y, o[2][1]);
      o[3][0] = fmaf(pp.w, vv[i].x, o[3][0]); o[3][1] = fmaf(pp.w, vv[i].y, o[3][1]);
    }
    __syncwarp();
  }
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    if (lane == 0) { s_m[warp][h] = m[h]; s_l[warp][h] = l[h]; }
    s_o[warp][h][2 * lane] = o[h][0];
    s_o[warp][h][2 * lane + 1] = o[h][1];
  }
  __syncthreads();
  // merge: warp w now finishes head w
  const int h = warp;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][h]);
  float L = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float mw = s_m[w][h];
    const float f = mw == -INFINITY ? 0.0f : expf(mw - M);  // warps without a tile hold nothing
    L = fmaf(s_l[w][h], f, L);
    o0 = fmaf(s_o[w][h][2 * lane], f, o0);
    o1 = fmaf(s_o[w][h][2 * lane + 1], f, o1);
  }
  const float inv = 1.0f / L;
  float* op = out + (size_t)t * q_dim + (size_t)(4 * g + h) * LE_HEAD_DIM + 2 * lane;
  *reinterpret_cast<float2*>(op) = make_float2(o0 * inv, o1 * inv);
}

// Greedy candidates of logits row blockIdx.y (ld floats apart) into part[row * gridDim.x + x].
__global__ void k_argmax_rows_batch(const float* __restrict__ logits, int vocab, size_t ld,
                                    ArgmaxPart* __restrict__ part) {
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  const float* row = logits + (size_t)blockIdx.y * ld;
  float bv = -1e30f;
  int bi = kNoIndex;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    argmax_offer(bv, bi, row[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) { s_bv[threadIdx.x >> 5] = bv; s_bi[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) argmax_merge(bv, bi, s_bv[w], s_bi[w]);
    part[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = ArgmaxPart{bv, bi};
  }
}

// result[row] = greedy id of row blockIdx.x from its nparts candidates (0 if none beats -1e30).
__global__ void k_argmax_finish_batch(const ArgmaxPart* __restrict__ part, int nparts, int32_t* __restrict__ result) {
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  const ArgmaxPart* pr = part + (size_t)blockIdx.x * nparts;
  float bv = -1e30f;
  int bi = kNoIndex;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) argmax_merge(bv, bi, pr[i].val, pr[i].idx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) { s_bv[threadIdx.x >> 5] = bv; s_bi[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) argmax_merge(bv, bi, s_bv[w], s_bi[w]);
    result[blockIdx.x] = bi == kNoIndex ? 0 : bi;
  }
}

}  // namespace le
