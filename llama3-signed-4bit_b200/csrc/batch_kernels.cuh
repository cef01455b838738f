// Token-batched kernels around the tensor-core GEMM (tc_gemm.cuh): embedding rows, decode
// attention for many (token, kv head) pairs, and per-row greedy argmax.  Each token carries its
// own sequence slot and position, so one launch serves batched decode (one token per sequence)
// and prefill (consecutive positions of one sequence; causality comes from each token reading
// the cache only up to its own position).
#pragma once

#include "decode_kernels.cuh"
#include "persistent.cuh"

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
// o = sum p v).  The token's own k / v are already in the cache (written by the RoPE / append
// kernel).  One CTA of 4 warps per (t, g): the CTA streams 32-position K / V tiles through shared
// memory (coalesced cp.async, double buffered, rows padded to 68 floats so that 16-byte row reads
// of 8 lanes hit distinct banks) and warp h computes q head h against each tile: lane = position
// for the scores, lane = dimension pair for p . v.  Softmax runs online (running max and sum,
// rescaled per tile).
//
// With gridDim.z = S > 1 the positions of each (t, g) are split into S contiguous ranges, one
// CTA each, and the CTA writes its unnormalised partial (running max m, sum l and o per head)
// to part[((t * kv_heads + g) * S + z)][4][66]; k_attn_combine merges them.
constexpr int kAttnPart = 4 * 66;
constexpr int kAttnRow = 68;
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(128)
    k_attn_batch(const float* __restrict__ q, int q_dim, const float* __restrict__ kc, const float* __restrict__ vc,
                 size_t slot_stride, int kv_dim, const int32_t* __restrict__ pos, const int32_t* __restrict__ slot,
                 float* __restrict__ out, float* __restrict__ part) {
  __shared__ __align__(16) float sk[2][32][kAttnRow];
  __shared__ __align__(16) float sv[2][32][kAttnRow];
  __shared__ float4 sp[4][32];  // per warp: this tile's softmax numerators (one head per warp)
  const int t = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = warp;
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
  auto load_tile = [&](int kt, int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = threadIdx.x + 128 * i;  // 16-byte chunk 0..511 of the tile
      const int r = c >> 4, d4 = c & 15;
      // rows past the range are masked out; read its last row in their place
      const size_t row = (size_t)min(kt * 32 + r, P - 1) * kv_dim + 4 * d4;
      cp_async16(smem_u32(&sk[buf][r][4 * d4]), Kb + row);
      cp_async16(smem_u32(&sv[buf][r][4 * d4]), Vb + row);
    }
    cp_async_commit();
  };
  float qv[64];
  {
    const float4* qp = reinterpret_cast<const float4*>(q + (size_t)t * q_dim + (size_t)(4 * g + h) * LE_HEAD_DIM);
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) {
      const float4 v = qp[d4];
      qv[4 * d4] = v.x; qv[4 * d4 + 1] = v.y; qv[4 * d4 + 2] = v.z; qv[4 * d4 + 3] = v.w;
    }
  }
  float m = -INFINITY, l = 0.0f, o0 = 0.0f, o1 = 0.0f;
  if (tile0 < tile1) load_tile(tile0, 0);
  for (int kt = tile0; kt < tile1; ++kt) {
    const int buf = (kt - tile0) & 1;
    if (kt + 1 < tile1) {
      load_tile(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // score of position kt*32 + lane for head h
    const float4* kr = reinterpret_cast<const float4*>(&sk[buf][lane][0]);
    float dot = 0.0f;
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) {
      const float4 k4 = kr[d4];
      dot = fmaf(qv[4 * d4], k4.x, dot);
      dot = fmaf(qv[4 * d4 + 1], k4.y, dot);
      dot = fmaf(qv[4 * d4 + 2], k4.z, dot);
      dot = fmaf(qv[4 * d4 + 3], k4.w, dot);
    }
    const float s = kt * 32 + lane < P ? dot * 0.125f : -INFINITY;
    const float mn = fmaxf(m, warp_max(s));  // finite: the tile holds a position of the range
    const float alpha = expf(m - mn);
    const float pe = expf(s - mn);
    l = l * alpha + warp_sum(pe);
    o0 *= alpha;
    o1 *= alpha;
    m = mn;
    reinterpret_cast<float*>(sp[h])[lane] = pe;
    __syncwarp();
    const float* pw = reinterpret_cast<const float*>(sp[h]);
#pragma unroll
    for (int j = 0; j < 32; ++j) {  // positions past the range have p = 0
      const float2 v2 = *reinterpret_cast<const float2*>(&sv[buf][j][2 * lane]);
      const float pj = pw[j];
      o0 = fmaf(pj, v2.x, o0);
      o1 = fmaf(pj, v2.y, o1);
    }
    __syncthreads();  // buffer buf is refilled by the next iteration's load
  }
  if (gridDim.z > 1) {
    float* pp = part + ((size_t)(t * gridDim.y + g) * gridDim.z + blockIdx.z) * kAttnPart + h * 66;
    if (lane == 0) { pp[0] = m; pp[1] = l; }
    pp[2 + 2 * lane] = o0;
    pp[3 + 2 * lane] = o1;
    return;
  }
  const float inv = 1.0f / l;
  float* op = out + (size_t)t * q_dim + (size_t)(4 * g + h) * LE_HEAD_DIM + 2 * lane;
  *reinterpret_cast<float2*>(op) = make_float2(o0 * inv, o1 * inv);
}

// Merges the S position-range partials of k_attn_batch: out = sum_z o_z e^(m_z - M) / sum_z
// l_z e^(m_z - M).  One CTA of 256 threads per token: thread = (head, dimension pair) slice.
__global__ void __launch_bounds__(256) k_attn_combine(const float* __restrict__ part, int kv_heads, int S,
                                                      int q_dim, float* __restrict__ out) {
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

// Causal attention of a prefill chunk: T consecutive tokens of one sequence (cache slot `slot`,
// positions p0 .. p0+T-1, all already in the cache).  Grid (kv heads, 32-token query tiles); one
// CTA per (kv head g, query tile):
// thread = (q head h = warp, token = lane), so a warp's lanes share every k / v element (shared-
// memory broadcast) and each thread keeps its own q row, o accumulator and online-softmax state
// (src/llama_engine.cpp:958-1021 per token: s = (q . k) * 0.125, softmax over 0..pos, o = sum p v).
// K / V tiles of 32 positions stream through shared memory with cp.async double buffering, each
// read once per 32 queries.
__global__ void __launch_bounds__(128, 2)
    k_attn_prefill(const float* __restrict__ q, int q_dim, const float* __restrict__ kc, const float* __restrict__ vc,
                   int kv_dim, int p0, int T, float* __restrict__ out) {
  __shared__ __align__(16) float sk[2][32][64];
  __shared__ __align__(16) float sv[2][32][64];
  const int g = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the last query tiles see the most keys: launch them first (blockIdx.y = 0 is dispatched
  // first) so the short ones fill the tail
  const int tok0 = (gridDim.y - 1 - blockIdx.y) * 32;
  const int t = min(tok0 + lane, T - 1);          // rows past T repeat the last token, unwritten
  const int pq = p0 + t;                          // this thread's query position
  const int p_last = p0 + min(tok0 + 31, T - 1);  // last position any thread of the CTA needs
  const int ntiles = p_last / 32 + 1;
  const float* Kb = kc + (size_t)g * LE_HEAD_DIM;
  const float* Vb = vc + (size_t)g * LE_HEAD_DIM;
  // tile loader: 32 rows x 256 bytes of k and of v, 128 threads x 4 x 16 bytes each
  auto load_tile = [&](int kt, int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = threadIdx.x + 128 * i;  // 16-byte chunk 0..511 of the tile
      const int r = c >> 4, d4 = c & 15;
      // rows past p_last are masked out; read the last needed row in their place
      const size_t row = (size_t)min(kt * 32 + r, p_last) * kv_dim + 4 * d4;
      cp_async16(smem_u32(&sk[buf][r][4 * d4]), Kb + row);
      cp_async16(smem_u32(&sv[buf][r][4 * d4]), Vb + row);
    }
    cp_async_commit();
  };
  float qv[64], o[64];
  {
    const float4* qp = reinterpret_cast<const float4*>(q + (size_t)t * q_dim + (size_t)(4 * g + warp) * LE_HEAD_DIM);
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) {
      const float4 v = qp[d4];
      qv[4 * d4] = v.x; qv[4 * d4 + 1] = v.y; qv[4 * d4 + 2] = v.z; qv[4 * d4 + 3] = v.w;
    }
  }
#pragma unroll
  for (int d = 0; d < 64; ++d) o[d] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  load_tile(0, 0);
  for (int kt = 0; kt < ntiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) {
      load_tile(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // 32 independent dot products (d outer, key inner), each still summed over d in order
    float sc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) sc[j] = 0.0f;
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float4 k4 = *reinterpret_cast<const float4*>(&sk[buf][j][4 * d4]);
        sc[j] = fmaf(qv[4 * d4], k4.x, sc[j]);
        sc[j] = fmaf(qv[4 * d4 + 1], k4.y, sc[j]);
        sc[j] = fmaf(qv[4 * d4 + 2], k4.z, sc[j]);
        sc[j] = fmaf(qv[4 * d4 + 3], k4.w, sc[j]);
      }
    }
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      sc[j] = kt * 32 + j <= pq ? sc[j] * 0.125f : -INFINITY;
      mt = fmaxf(mt, sc[j]);
    }
    // tile 0 always holds position 0 <= pq, so m is finite from the first tile on
    const float mn = fmaxf(m, mt);
    const float alpha = expf(m - mn);
    float ls = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      sc[j] = expf(sc[j] - mn);
      ls += sc[j];
    }
    l = l * alpha + ls;
    m = mn;
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] *= alpha;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float4* vr = reinterpret_cast<const float4*>(&sv[buf][j][0]);
#pragma unroll
      for (int d4 = 0; d4 < 16; ++d4) {
        const float4 v4 = vr[d4];
        o[4 * d4] = fmaf(sc[j], v4.x, o[4 * d4]);
        o[4 * d4 + 1] = fmaf(sc[j], v4.y, o[4 * d4 + 1]);
        o[4 * d4 + 2] = fmaf(sc[j], v4.z, o[4 * d4 + 2]);
        o[4 * d4 + 3] = fmaf(sc[j], v4.w, o[4 * d4 + 3]);
      }
    }
    __syncthreads();  // buffer buf is refilled by the next iteration's load
  }
  if (tok0 + lane < T) {
    const float inv = 1.0f / l;
    float4* op = reinterpret_cast<float4*>(out + (size_t)t * q_dim + (size_t)(4 * g + warp) * LE_HEAD_DIM);
#pragma unroll
    for (int d4 = 0; d4 < 16; ++d4)
      op[d4] = make_float4(o[4 * d4] * inv, o[4 * d4 + 1] * inv, o[4 * d4 + 2] * inv, o[4 * d4 + 3] * inv);
  }
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
