// Token-batched kernels around the tensor-core GEMM (tc_gemm.cuh): embedding rows, decode
// attention for many (token, kv head) pairs, and per-row greedy argmax.  Each token carries its
// own sequence slot and position, so one launch serves batched decode (one token per sequence)
// and prefill (consecutive positions of one sequence; causality comes from each token reading
// the cache only up to its own position).
#pragma once

#include <cuda_bf16.h>

#include "decode_kernels.cuh"
#include "persistent.cuh"
#include "tc_gemm.cuh"

namespace le {

// x[t] = dequantised row tok[t] of the tied lm_head (dequantize_embedding_row,
// src/llama_engine.cpp:182-220).
__global__ void k_embed_batch(QMat E, const int32_t* __restrict__ tok, float* __restrict__ x, int ldx) {
  grid_dep_begin();
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
// o = sum p v).  With qkv == nullptr, q comes rotated in `q` and the token's own k / v are
// already in the cache (RoPE / append kernel).  With qkv set, the CTA builds them itself from
// the q | k | v GEMM output (the sum of its nsplit split-K planes, rotated with the RoPE table
// as in k_rope_append, src/llama_engine.cpp:953-956), uses the token's k / v for position pos
// in place of the cache row, and the CTA whose range holds pos appends them to the cache.  One CTA of 4 warps per (t, g): the CTA streams 32-position K / V tiles through shared
// memory (coalesced cp.async, three tiles in a ring, rows padded to 68 floats so that 16-byte row
// reads of 8 lanes hit distinct banks), one barrier per tile.  Warp w owns positions 8w .. 8w+7
// of every tile: lane (j, h) = 4j + h holds q of head h and computes the whole 64-wide score of
// position 8w + j; each warp keeps its own online softmax per head (running max and sum,
// rescaled per tile) and o for dimensions 2 lane, 2 lane + 1 of the four heads (p . v with the
// probabilities broadcast by shuffles); the four warps' (max, sum, o) are merged at the end.
//
// With gridDim.z = S > 1 the positions of each (t, g) are split into S contiguous ranges, one
// CTA each, and the CTA writes its unnormalised partial (running max m, sum l and o per head)
// to part[((t * kv_heads + g) * S + z)][4][66]; k_attn_combine merges them.
constexpr int kAttnPart = 4 * 66;
constexpr int kAttnRow = 68;
constexpr int kAttnSmem = 2 * 3 * 32 * kAttnRow * 4;  // dynamic shared memory of k_attn_batch
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float attn_sum_planes(const float* p, int nsplit, size_t stride) {
  return tc::sum_planes(p, nsplit, stride);
}

__global__ void __launch_bounds__(128, 4)
    k_attn_batch(const float* __restrict__ q, int q_dim, float* __restrict__ kc, float* __restrict__ vc,
                 size_t slot_stride, int kv_dim, const int32_t* __restrict__ pos, const int32_t* __restrict__ slot,
                 float* __restrict__ out, float* __restrict__ part, const float* __restrict__ qkv, int nsplit,
                 size_t split_stride, const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                 uint8_t* __restrict__ img) {
  grid_dep_begin();
  // three-stage ring of K / V tiles (two tiles in flight while one is used)
  extern __shared__ __align__(16) float attn_smem[];
  float (*sk)[32][kAttnRow] = reinterpret_cast<float (*)[32][kAttnRow]>(attn_smem);
  float (*sv)[32][kAttnRow] = reinterpret_cast<float (*)[32][kAttnRow]>(attn_smem + 3 * 32 * kAttnRow);
  __shared__ float wm[4][4], wl[4][4];         // per warp and head: running max and sum
  __shared__ __align__(16) float sqkv[6][64];  // with qkv: q of the 4 heads, k and v of this token
  __shared__ float sbs[4];                     // with img: per warp, the sum of its head's outputs
  const int t = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P_all = pos[t] + 1;
  // this CTA's position range [tile0 * 32, P): whole 32-position tiles, split z of gridDim.z
  const int tiles = (P_all + 31) >> 5;
  const int per = (tiles + gridDim.z - 1) / gridDim.z;
  const int tile0 = per * blockIdx.z;
  const int P = min(P_all, (tile0 + per) * 32);
  const int tile1 = (P + 31) >> 5;  // one past the last tile
  const size_t base = (size_t)slot[t] * slot_stride + (size_t)g * LE_HEAD_DIM;
  const float* Kb = kc + base;
  const float* Vb = vc + base;
  const int p_tok = P_all - 1;
  if (qkv != nullptr) {  // rows: q heads 4g .. 4g+3, k head g, v head g
    const float* row = qkv + (size_t)t * (q_dim + 2 * kv_dim);
    for (int j = threadIdx.x; j < 5 * 32 + 64; j += blockDim.x) {
      if (j < 5 * 32) {  // rotated pair (i, i + 32) of q head j / 32 (4 = the k head)
        const int hh = j >> 5, i = j & 31;
        const int off = hh < 4 ? (4 * g + hh) * LE_HEAD_DIM + i : q_dim + g * LE_HEAD_DIM + i;
        const float c = rope_cos[p_tok * 32 + i], sn = rope_sin[p_tok * 32 + i];
        const float r0 = attn_sum_planes(row + off, nsplit, split_stride);
        const float r1 = attn_sum_planes(row + off + 32, nsplit, split_stride);
        sqkv[hh][i] = __fsub_rn(__fmul_rn(r0, c), __fmul_rn(r1, sn));
        sqkv[hh][i + 32] = __fadd_rn(__fmul_rn(r0, sn), __fmul_rn(r1, c));
      } else {
        const int e = j - 5 * 32;
        sqkv[5][e] = attn_sum_planes(row + q_dim + kv_dim + g * LE_HEAD_DIM + e, nsplit, split_stride);
      }
    }
    __syncthreads();
  }
  auto load_tile = [&](int kt, int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = threadIdx.x + 128 * i;  // 16-byte chunk 0..511 of the tile
      const int r = c >> 4, d4 = c & 15;
      // rows past the range are masked out of the scores; their K is the range's last row, and
      // their V is zero, so that no value left in the cache beyond the range reaches p . v
      const size_t row = (size_t)min(kt * 32 + r, P - 1) * kv_dim + 4 * d4;
      cp_async16(smem_u32(&sk[buf][r][4 * d4]), Kb + row);
      if (kt * 32 + r < P) cp_async16(smem_u32(&sv[buf][r][4 * d4]), Vb + row);
      else *reinterpret_cast<float4*>(&sv[buf][r][4 * d4]) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
  };
  // q of this lane's head, all 64 dimensions (lane = 4 x position-in-warp + head)
  const int hq = lane & 3, pw = lane >> 2;
  float qv[64];
  {
    const float* qt = qkv != nullptr ? &sqkv[hq][0] : q + (size_t)t * q_dim + (size_t)(4 * g + hq) * LE_HEAD_DIM;
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) {
      const float4 v = reinterpret_cast<const float4*>(qt)[d4];
      qv[4 * d4] = v.x; qv[4 * d4 + 1] = v.y; qv[4 * d4 + 2] = v.z; qv[4 * d4 + 3] = v.w;
    }
  }
  // this warp's online softmax of head hq (the same in the 8 lanes of the head) and its p . v for
  // dimensions 2 lane, 2 lane + 1 of the four heads
  float m = -INFINITY, l = 0.0f;
  float o[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
  if (tile0 < tile1) load_tile(tile0, 0);
  if (tile0 + 1 < tile1) load_tile(tile0 + 1, 1);
  for (int kt = tile0; kt < tile1; ++kt) {
    const int buf = (kt - tile0) % 3;
    if (kt + 1 < tile1) cp_async_wait<1>();
    else cp_async_wait<0>();
    __syncthreads();  // tile kt has landed for every thread, and tile kt - 1's buffer is free
    if (kt + 2 < tile1) load_tile(kt + 2, (kt - tile0 + 2) % 3);
    if (qkv != nullptr && p_tok >= kt * 32 && p_tok < kt * 32 + 32) {  // this step's own k / v
      const int r = p_tok - kt * 32;
      if (threadIdx.x < 64) sk[buf][r][threadIdx.x] = sqkv[4][threadIdx.x];
      else sv[buf][r][threadIdx.x - 64] = sqkv[5][threadIdx.x - 64];
      __syncthreads();
    }
    // score of position kt*32 + 8 warp + pw for head hq
    const int r = 8 * warp + pw;
    const float4* kr = reinterpret_cast<const float4*>(&sk[buf][r][0]);
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) {
      const float4 k4 = kr[d4];
      d0 = fmaf(qv[4 * d4], k4.x, d0);
      d1 = fmaf(qv[4 * d4 + 1], k4.y, d1);
      d2 = fmaf(qv[4 * d4 + 2], k4.z, d2);
      d3 = fmaf(qv[4 * d4 + 3], k4.w, d3);
    }
    const float s = kt * 32 + r < P ? ((d0 + d1) + (d2 + d3)) * 0.125f : -INFINITY;
    // the warp's 8 positions of head hq sit in lanes hq, hq + 4, ..., hq + 28
    float tmax = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 4));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
    const float mn = fmaxf(m, tmax);
    const float alpha = mn == -INFINITY ? 1.0f : expf(m - mn);  // no position of the head yet
    const float pe = s == -INFINITY ? 0.0f : expf(s - mn);
    float psum = pe + __shfl_xor_sync(0xffffffffu, pe, 4);
    psum += __shfl_xor_sync(0xffffffffu, psum, 8);
    psum += __shfl_xor_sync(0xffffffffu, psum, 16);
    l = l * alpha + psum;
    m = mn;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float ah = __shfl_sync(0xffffffffu, alpha, h);
      o[h][0] *= ah;
      o[h][1] *= ah;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 v2 = *reinterpret_cast<const float2*>(&sv[buf][8 * warp + j][2 * lane]);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float pj = __shfl_sync(0xffffffffu, pe, 4 * j + h);
        o[h][0] = fmaf(pj, v2.x, o[h][0]);
        o[h][1] = fmaf(pj, v2.y, o[h][1]);
      }
    }
  }
  __syncthreads();  // every warp is done with the ring: its memory now holds the warps' o
  float* wo = attn_smem;  // [warp][head][64]
  if (lane < 4) {  // lane h (position 0) holds head h's max and sum
    wm[warp][lane] = m;
    wl[warp][lane] = l;
  }
#pragma unroll
  for (int h = 0; h < 4; ++h)
    *reinterpret_cast<float2*>(&wo[(warp * 4 + h) * 64 + 2 * lane]) = make_float2(o[h][0], o[h][1]);
  if (qkv != nullptr && p_tok >= tile0 * 32 && p_tok < P) {  // append k / v at (slot, pos)
    const size_t crow = base + (size_t)p_tok * kv_dim;
    if (threadIdx.x < 64) kc[crow + threadIdx.x] = sqkv[4][threadIdx.x];
    else vc[crow + threadIdx.x - 64] = sqkv[5][threadIdx.x - 64];
  }
  __syncthreads();
  // merge of the four warps: thread = (head ph = warp, dimensions 2 dp, 2 dp + 1)
  const int ph = warp, dp = lane;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][ph]);
  float L = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float f = wm[w][ph] == -INFINITY ? 0.0f : expf(wm[w][ph] - M);  // warps without positions
    const float2 ow = *reinterpret_cast<const float2*>(&wo[(w * 4 + ph) * 64 + 2 * dp]);
    L = fmaf(wl[w][ph], f, L);
    o0 = fmaf(ow.x, f, o0);
    o1 = fmaf(ow.y, f, o1);
  }
  if (gridDim.z > 1) {
    float* pp = part + ((size_t)(t * gridDim.y + g) * gridDim.z + blockIdx.z) * kAttnPart + ph * 66;
    if (dp == 0) { pp[0] = M; pp[1] = L; }
    pp[2 + 2 * dp] = o0;
    pp[3 + 2 * dp] = o1;
    return;
  }
  const float inv = 1.0f / L;
  const float a0 = o0 * inv, a1 = o1 * inv;
  if (img != nullptr) {
    // the o-proj GEMM input, written directly in the k_tc_stage image layout: bf16 hi / lo parts
    // of the element pair at its place in the 8-element run, and the 128-block sums
    const __nv_bfloat162 hh = __floats2bfloat162_rn(a0, a1);
    const __nv_bfloat162 ll = __floats2bfloat162_rn(a0 - __low2float(hh), a1 - __high2float(hh));
    const int e = (4 * g + ph) * LE_HEAD_DIM + 2 * dp;
    const int i0 = e & ~7, j = (e & 7) >> 1;
    const int tt = t / tc::kTok, tr = t % tc::kTok, kbt = q_dim >> 7;
    const int kb = i0 >> 7, kk = i0 & 127, atom = kk >> 6, c = (kk & 63) >> 3;
    uint8_t* im = img + ((size_t)tt * kbt + kb) * tc::kImgBytes;
    const size_t off = (size_t)atom * 2 * tc::kAtom + tr * 128 + ((c ^ (tr & 7)) << 4) + 4 * j;
    *reinterpret_cast<__nv_bfloat162*>(im + off) = hh;
    *reinterpret_cast<__nv_bfloat162*>(im + tc::kAtom + off) = ll;
    // block 2g holds heads 4g, 4g+1 (warps 0, 1), block 2g+1 heads 4g+2, 4g+3 (warps 2, 3)
    float bs = a0 + a1;
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o2);
    if (lane == 0) sbs[warp] = bs;
    __syncthreads();
    if (threadIdx.x < 2) {
      const int b = threadIdx.x;
      reinterpret_cast<float*>(img + ((size_t)tt * kbt + 2 * g + b) * tc::kImgBytes + tc::kOffXs)[tr] =
          sbs[2 * b] + sbs[2 * b + 1];
    }
    return;
  }
  float* op = out + (size_t)t * q_dim + (size_t)(4 * g + ph) * LE_HEAD_DIM + 2 * dp;
  *reinterpret_cast<float2*>(op) = make_float2(a0, a1);
}

// Merges the S position-range partials of k_attn_batch: out = sum_z o_z e^(m_z - M) / sum_z
// l_z e^(m_z - M).  One CTA of 256 threads per token: thread = (head, dimension pair) slice.
__global__ void __launch_bounds__(256) k_attn_combine(const float* __restrict__ part, int kv_heads, int S,
                                                      int q_dim, float* __restrict__ out) {
  grid_dep_begin();
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < kv_heads * 4 * 32; i += blockDim.x) {
    const int g = i >> 7, h = (i >> 5) & 3, dp = i & 31;
    const float* pp = part + (size_t)(t * kv_heads + g) * S * kAttnPart + h * 66;
    float M = -INFINITY;
    for (int z = 0; z < S; ++z) M = fmaxf(M, pp[(size_t)z * kAttnPart]);
    float L = 0.0f, o0 = 0.0f, o1 = 0.0f;
    for (int z = 0; z < S; ++z) {
      const float* pz = pp + (size_t)z * kAttnPart;
      const float mz = pz[0];
      const float f = mz == -INFINITY ? 0.0f : expf(mz - M);  // ranges past the token's position
      L = fmaf(pz[1], f, L);
      o0 = fmaf(pz[2 + 2 * dp], f, o0);
      o1 = fmaf(pz[3 + 2 * dp], f, o1);
    }
    const float inv = 1.0f / L;
    float* op = out + (size_t)t * q_dim + (size_t)(4 * g + h) * LE_HEAD_DIM + 2 * dp;
    *reinterpret_cast<float2*>(op) = make_float2(o0 * inv, o1 * inv);
  }
}

// bf16 hi / lo parts of fp32 values for the tensor cores: x = hi + lo with hi = bf16(x) and
// lo = bf16(x - hi), so a product of two such sums, taken as hi.hi + hi.lo + lo.hi, carries
// ~2^-16 relative error at most.
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// hi / lo split of a pair: hi = bf16(x), lo = bf16(x - hi)
__device__ __forceinline__ void split_bf16(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack_bf16(a - __low2float(h), b - __high2float(h));
}

// Greedy candidates of logits row blockIdx.y (ld floats apart) into part[row * gridDim.x + x].
__global__ void k_argmax_rows_batch(const float* __restrict__ logits, int vocab, size_t ld,
                                    ArgmaxPart* __restrict__ part) {
  grid_dep_begin();
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

// Log-probability of a target id under one logits row (the lm-eval consumer's formula,
// tests/lm_eval_adapter.py:175-181: (l[t] - max) - log(sum exp(l - max))) and whether the target
// is the greedy id (first index among equal maxima).  One CTA of 1024 threads per row; rows with
// target < 0 are skipped.
__global__ void __launch_bounds__(1024) k_logprob_rows(const float* __restrict__ logits, int vocab, size_t ld,
                                                       const int32_t* __restrict__ target,
                                                       float* __restrict__ out_lp, int32_t* __restrict__ out_greedy) {
  grid_dep_begin();
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  __shared__ float s_sum[32];
  const int row = blockIdx.x;
  const int tgt = target[row];
  if (tgt < 0) return;
  const float* l = logits + (size_t)row * ld;
  float bv = -INFINITY;
  int bi = kNoIndex;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = l[i];
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { s_v[wid] = bv; s_i[wid] = bi; }
  __syncthreads();
  if (wid == 0) {
    bv = lane < (int)(blockDim.x >> 5) ? s_v[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? s_i[lane] : kNoIndex;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { s_v[0] = bv; s_i[0] = bi; }
  }
  __syncthreads();
  const float mx = s_v[0];
  float se = 0.0f;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) se += expf(l[i] - mx);
  se = warp_sum(se);
  if (lane == 0) s_sum[wid] = se;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += s_sum[w];
    out_lp[row] = (l[tgt] - mx) - logf(tot);
    if (out_greedy) out_greedy[row] = s_i[0] == tgt ? 1 : 0;
  }
}

// result[row] = greedy id of row blockIdx.x from its nparts candidates (0 if none beats -1e30).
__global__ void k_argmax_finish_batch(const ArgmaxPart* __restrict__ part, int nparts, int32_t* __restrict__ result) {
  grid_dep_begin();
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
