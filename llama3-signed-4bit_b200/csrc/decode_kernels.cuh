// Decode-step kernels for the block-128 4-bit LLaMA token loop (sm_100a).
//
// One token step (src/llama_engine.cpp:935-1042) runs as
//   embed -> L x { qkv (rmsnorm prologue) -> attention (RoPE, KV append) -> o-proj (+residual)
//                  -> gate/up (rmsnorm prologue, SiLU*up epilogue) -> down (+residual) }
//   -> lm_head (rmsnorm prologue, per-CTA argmax) -> argmax finish
// captured once into a CUDA graph.  Token and position are read from device memory, so the
// same graph serves every step.
#pragma once

#include "common.cuh"

namespace le {

// Per-step parameters read by the graph's kernels.
struct StepParams {
  int32_t token;  // input token of this step (already range-checked)
  int32_t pos;    // position of this step
  int32_t step;   // index into the device token log (device-resident greedy loop)
  int32_t pad;
};

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// ---------------------------------------------------------------------------------------------
// Prologues: the activation vector(s) of a GEMV are staged in shared memory together with their
// 128-wide block sums (compute_x_block_sums, src/llama_engine.cpp:496-521).
// ---------------------------------------------------------------------------------------------

// xs[i] = x[i] * w[i] * inv,  inv = 1 / sqrt(sum(x^2)/n + 1e-5)   (rms_norm, :87-115)
__device__ __forceinline__ void stage_rmsnorm(const float* __restrict__ x, const float* __restrict__ w,
                                              float* xs, int n, float* red) {
  float ss = 0.0f;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(x + i);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)n + 1e-5f);
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(x + i);
    float4 g = *reinterpret_cast<const float4*>(w + i);
    float4 o;
    o.x = __fmul_rn(__fmul_rn(v.x, g.x), inv);
    o.y = __fmul_rn(__fmul_rn(v.y, g.y), inv);
    o.z = __fmul_rn(__fmul_rn(v.z, g.z), inv);
    o.w = __fmul_rn(__fmul_rn(v.w, g.w), inv);
    *reinterpret_cast<float4*>(xs + i) = o;
  }
}

__device__ __forceinline__ void stage_copy(const float* __restrict__ x, float* xs, int n) {
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
    *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
}

// bsum[b] = sum of xs[128b .. 128b+127]; one warp per block.
__device__ __forceinline__ void stage_block_sums(const float* xs, float* bsum, int n) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int b = wid; b < n / 128; b += nw) {
    float4 v = *reinterpret_cast<const float4*>(xs + b * 128 + lane * 4);
    float s = (v.x + v.y) + (v.z + v.w);
    s = warp_sum(s);
    if (lane == 0) bsum[b] = s;
  }
}

// ---------------------------------------------------------------------------------------------
// Warp GEMV core.
//
// A warp computes R consecutive output rows for MX activation vectors.  A row of K weights is
// K/2 bytes of nibbles, read as 16-byte chunks: lane l takes chunks l, l+32, ... (coalesced
// 512-byte warp loads).  A chunk holds 32 consecutive weights, a quarter of a 128-block.  The
// factored form of the reference (src/llama_engine.cpp:231-232, 315-319)
//     y = sum_b  min_b * xs_b  +  step_b * sum_k q_k x_k
// is applied per chunk: the lane multiplies its chunk's q.x partial by step_b, and the lane
// owning the first chunk of block b adds min_b * xs_b.  A warp reduction finishes the row.
// All weight loads of the warp's rows are issued before any arithmetic.
// ---------------------------------------------------------------------------------------------
template <int MX, int R, int CPL>
__device__ __forceinline__ void warp_gemv(const QMat& W, int row0, const float* xs, int x_stride,
                                          const float* bsum, int bs_stride, float (&out)[MX][R]) {
  const int lane = threadIdx.x & 31;
  const int nchunks = W.K >> 5;
  const int nb = W.K >> 7;
  float acc[MX][R];
#pragma unroll
  for (int m = 0; m < MX; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[m][r] = 0.0f;

  for (int base = 0; base < nchunks; base += 32 * CPL) {
    uint4 w[R][CPL];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint8_t* rowp = W.nib + (size_t)(row0 + r) * (W.K >> 1);
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int c = base + lane + 32 * i;
        if (c < nchunks) w[r][i] = ld_stream_u4(rowp + (size_t)c * 16);
        else w[r][i] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = base + lane + 32 * i;
      if (c < nchunks) {
        const int b = c >> 2;
        float dot[MX][R];
#pragma unroll
        for (int m = 0; m < MX; ++m)
#pragma unroll
          for (int r = 0; r < R; ++r) dot[m][r] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float xv[MX][8];
#pragma unroll
          for (int m = 0; m < MX; ++m) {
            const float4 a = *reinterpret_cast<const float4*>(xs + m * x_stride + c * 32 + j * 8);
            const float4 bq = *reinterpret_cast<const float4*>(xs + m * x_stride + c * 32 + j * 8 + 4);
            xv[m][0] = a.x; xv[m][1] = a.y; xv[m][2] = a.z; xv[m][3] = a.w;
            xv[m][4] = bq.x; xv[m][5] = bq.y; xv[m][6] = bq.z; xv[m][7] = bq.w;
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint32_t v = j == 0 ? w[r][i].x : j == 1 ? w[r][i].y : j == 2 ? w[r][i].z : w[r][i].w;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const float q = nib_to_f32((v >> (4 * t)) & 0xFu);
#pragma unroll
              for (int m = 0; m < MX; ++m) dot[m][r] = fmaf(q, xv[m][t], dot[m][r]);
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const size_t blk = (size_t)(row0 + r) * nb + b;
          const float st = bf16_bits_to_f32(__ldg(W.step + blk));
          const float mv = bf16_bits_to_f32(__ldg(W.mn + blk));
#pragma unroll
          for (int m = 0; m < MX; ++m) {
            float t = st * dot[m][r];
            if ((c & 3) == 0) t = fmaf(mv, bsum[m * bs_stride + b], t);
            acc[m][r] += t;
          }
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MX; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) out[m][r] = warp_sum(acc[m][r]);
}

// ---------------------------------------------------------------------------------------------
// Embedding: x = row `token` of the tied lm_head, dequantised (dequantize_embedding_row,
// src/llama_engine.cpp:182-220).  Plain multiply then add, as in the reference.
// ---------------------------------------------------------------------------------------------
__global__ void k_embed(QMat E, const StepParams* __restrict__ prm, const int32_t* __restrict__ tok_override,
                        float* __restrict__ out) {
  const int token = tok_override ? *tok_override : prm->token;
  const int K = E.K, nb = K >> 7;
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

// ---------------------------------------------------------------------------------------------
// QKV: rmsnorm(x, in_norm) prologue, then the rows of Wq, Wk, Wv (one concatenated row space).
// Output: raw (un-rotated) q | k | v.
// ---------------------------------------------------------------------------------------------
template <int R>
__global__ void __launch_bounds__(kThreads) k_qkv(const float* __restrict__ x, const float* __restrict__ gnorm,
                                                  QMat Wq, QMat Wk, QMat Wv, float* __restrict__ qkv) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const int K = Wq.K;
  float* bsum = xs + K;
  float* red = bsum + K / 128;
  stage_rmsnorm(x, gnorm, xs, K, red);
  __syncthreads();
  stage_block_sums(xs, bsum, K);
  __syncthreads();
  const int nq = Wq.N, nk = Wk.N, total = Wq.N + Wk.N + Wv.N;
  const int lane = threadIdx.x & 31;
  for (int g = blockIdx.x * kWarps + (threadIdx.x >> 5); g * R < total; g += gridDim.x * kWarps) {
    const int gr = g * R;
    const QMat& W = gr < nq ? Wq : (gr < nq + nk ? Wk : Wv);
    const int row0 = gr < nq ? gr : (gr < nq + nk ? gr - nq : gr - nq - nk);
    float out[1][R];
    warp_gemv<1, R, 2>(W, row0, xs, K, bsum, 0, out);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) qkv[gr + r] = out[0][r];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Attention for one token (src/llama_engine.cpp:953-1021): RoPE on q and the new k
// (apply_rope, :120-151, table lookup), K/V append at `pos`, then per q-head softmax attention
// over positions 0..pos of its kv head (kv_h = h / (heads/kv_heads)).  One CTA per q head.
// Every CTA rotates the new k itself and uses that copy for t == pos; the first q head of each
// kv group also stores it into the cache, so no CTA reads a cache row another CTA is writing.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_attention(const float* __restrict__ qkv, float* __restrict__ kc,
                                                        float* __restrict__ vc, const float* __restrict__ rope_cos,
                                                        const float* __restrict__ rope_sin,
                                                        const StepParams* __restrict__ prm, int n_heads,
                                                        int n_kv_heads, float* __restrict__ attn_out) {
  extern __shared__ float4 smem4[];
  float* sq = reinterpret_cast<float*>(smem4);  // 64
  float* sk = sq + 64;                          // 64
  float* sv = sk + 64;                          // 64
  float* red = sv + 64;                         // 32
  float* pv = red + 32;                         // 4 x 64
  float* scores = pv + 256;                     // pos+1
  const int h = blockIdx.x;
  const int group = n_heads / n_kv_heads;
  const int kvh = h / group;
  const int kv_dim = n_kv_heads * LE_HEAD_DIM;
  const int q_dim = n_heads * LE_HEAD_DIM;
  const int pos = prm->pos;
  const int tid = threadIdx.x;

  if (tid < 32) {
    const float c = rope_cos[pos * 32 + tid], s = rope_sin[pos * 32 + tid];
    const float* qh = qkv + h * LE_HEAD_DIM;
    const float r0 = qh[tid], r1 = qh[tid + 32];
    sq[tid] = __fsub_rn(__fmul_rn(r0, c), __fmul_rn(r1, s));
    sq[tid + 32] = __fadd_rn(__fmul_rn(r0, s), __fmul_rn(r1, c));
  } else if (tid < 64) {
    const int i = tid - 32;
    const float c = rope_cos[pos * 32 + i], s = rope_sin[pos * 32 + i];
    const float* kh = qkv + q_dim + kvh * LE_HEAD_DIM;
    const float r0 = kh[i], r1 = kh[i + 32];
    sk[i] = __fsub_rn(__fmul_rn(r0, c), __fmul_rn(r1, s));
    sk[i + 32] = __fadd_rn(__fmul_rn(r0, s), __fmul_rn(r1, c));
  } else if (tid < 128) {
    const int d = tid - 64;
    sv[d] = qkv[q_dim + kv_dim + kvh * LE_HEAD_DIM + d];
  }
  __syncthreads();
  if (h % group == 0 && tid < 64) {
    kc[(size_t)pos * kv_dim + kvh * LE_HEAD_DIM + tid] = sk[tid];
    vc[(size_t)pos * kv_dim + kvh * LE_HEAD_DIM + tid] = sv[tid];
  }

  // scores s_t = (q . k_t) * 0.125
  float mx = -INFINITY;
  for (int t = tid; t <= pos; t += blockDim.x) {
    const float* kt = t == pos ? sk : kc + (size_t)t * kv_dim + kvh * LE_HEAD_DIM;
    float dot = 0.0f;
#pragma unroll
    for (int d = 0; d < LE_HEAD_DIM; d += 4) {
      const float4 kv4 = *reinterpret_cast<const float4*>(kt + d);
      dot = fmaf(sq[d], kv4.x, dot);
      dot = fmaf(sq[d + 1], kv4.y, dot);
      dot = fmaf(sq[d + 2], kv4.z, dot);
      dot = fmaf(sq[d + 3], kv4.w, dot);
    }
    const float s = dot * 0.125f;
    scores[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_max(mx, red);
  float se = 0.0f;
  for (int t = tid; t <= pos; t += blockDim.x) {
    const float e = expf(scores[t] - mx);
    scores[t] = e;
    se += e;
  }
  se = block_sum(se, red);
  const float inv = 1.0f / se;
  __syncthreads();
  // out[d] = sum_t (e_t * inv) * v_t[d]; 4 position groups of 64 threads
  const int d = tid & 63, tg = tid >> 6;
  float acc = 0.0f;
  for (int t = tg; t <= pos; t += 4) {
    const float vt = t == pos ? sv[d] : vc[(size_t)t * kv_dim + kvh * LE_HEAD_DIM + d];
    acc = fmaf(scores[t] * inv, vt, acc);
  }
  pv[tg * 64 + d] = acc;
  __syncthreads();
  if (tid < 64) attn_out[h * LE_HEAD_DIM + tid] = (pv[tid] + pv[64 + tid]) + (pv[128 + tid] + pv[192 + tid]);
}

// ---------------------------------------------------------------------------------------------
// Projection with residual: x[n] += W[n,:] . a   (o-proj at :1024-1025, down at :1033-1034).
// The input vector a (K floats) is staged with its block sums.
// ---------------------------------------------------------------------------------------------
template <int R, int CPL>
__global__ void __launch_bounds__(kThreads) k_proj_residual(const float* __restrict__ a, QMat W, float* __restrict__ x) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const int K = W.K;
  float* bsum = xs + K;
  stage_copy(a, xs, K);
  __syncthreads();
  stage_block_sums(xs, bsum, K);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int g = blockIdx.x * kWarps + (threadIdx.x >> 5); g * R < W.N; g += gridDim.x * kWarps) {
    float out[1][R];
    warp_gemv<1, R, CPL>(W, g * R, xs, K, bsum, 0, out);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) x[g * R + r] += out[0][r];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Gate/up with SwiGLU epilogue: act[n] = silu(g_n) * u_n, silu(v) = v / (1 + exp(-v))
// (signed_4bit_b128_fused_swiglu, src/llama_engine.cpp:362-491).  rmsnorm(x, post_norm) prologue.
// ---------------------------------------------------------------------------------------------
template <int R>
__global__ void __launch_bounds__(kThreads) k_gateup(const float* __restrict__ x, const float* __restrict__ gnorm,
                                                     QMat Wg, QMat Wu, float* __restrict__ act) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const int K = Wg.K;
  float* bsum = xs + K;
  float* red = bsum + K / 128;
  stage_rmsnorm(x, gnorm, xs, K, red);
  __syncthreads();
  stage_block_sums(xs, bsum, K);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int g = blockIdx.x * kWarps + (threadIdx.x >> 5); g * R < Wg.N; g += gridDim.x * kWarps) {
    float go[1][R], uo[1][R];
    warp_gemv<1, R, 2>(Wg, g * R, xs, K, bsum, 0, go);
    warp_gemv<1, R, 2>(Wu, g * R, xs, K, bsum, 0, uo);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float gv = go[0][r];
        act[g * R + r] = (gv / (1.0f + expf(-gv))) * uo[0][r];
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// lm_head: rmsnorm(x, final_norm) prologue, logits[n] = W[n,:] . xs (src/llama_engine.cpp:1037-1041),
// plus the CTA's greedy candidate: the first index among its maxima (sample_top_p greedy branch,
// :785-792: strict '>' from -1e30, so the lowest index wins ties and NaN never wins).
// ---------------------------------------------------------------------------------------------
struct ArgmaxPart {
  float val;
  int32_t idx;
};

// Candidates are (value, index) pairs; (-1e30, INT_MAX) is the identity.  A logit enters only
// if it is > -1e30 (so NaN and -inf never win); among equal values the lower index wins.
constexpr int kNoIndex = 0x7fffffff;
__device__ __forceinline__ void argmax_merge(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}
__device__ __forceinline__ void argmax_offer(float& bv, int& bi, float v, int i) {
  if (v > -1e30f) argmax_merge(bv, bi, v, i);
}

template <int R>
__global__ void __launch_bounds__(kThreads) k_lmhead(const float* __restrict__ x, const float* __restrict__ gnorm,
                                                     QMat W, float* __restrict__ logits, ArgmaxPart* __restrict__ part) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const int K = W.K;
  float* bsum = xs + K;
  float* red = bsum + K / 128;
  __shared__ float s_bv[kWarps];
  __shared__ int s_bi[kWarps];
  stage_rmsnorm(x, gnorm, xs, K, red);
  __syncthreads();
  stage_block_sums(xs, bsum, K);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  float bv = -1e30f;
  int bi = kNoIndex;
  for (int g = blockIdx.x * kWarps + (threadIdx.x >> 5); g * R < W.N; g += gridDim.x * kWarps) {
    float out[1][R];
    warp_gemv<1, R, 2>(W, g * R, xs, K, bsum, 0, out);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        logits[g * R + r] = out[0][r];
        argmax_offer(bv, bi, out[0][r], g * R + r);
      }
    }
  }
  if (lane == 0) { s_bv[threadIdx.x >> 5] = bv; s_bi[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kWarps; ++w) argmax_merge(bv, bi, s_bv[w], s_bi[w]);
    part[blockIdx.x] = ArgmaxPart{bv, bi};
  }
}

// Reduces the per-CTA candidates.  Writes the greedy id to *result (0 when no logit exceeds
// -1e30, as the reference).  With `advance`, also appends it to the device token log and moves
// the step parameters to (token = id, pos + 1) for the next graph launch.
__global__ void k_argmax_finish(const ArgmaxPart* __restrict__ part, int nparts, int32_t* __restrict__ result,
                                StepParams* __restrict__ prm, int32_t* __restrict__ token_log, int advance) {
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  float bv = -1e30f;
  int bi = kNoIndex;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) argmax_merge(bv, bi, part[i].val, part[i].idx);
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
    const int id = bi == kNoIndex ? 0 : bi;
    *result = id;
    if (advance) {
      token_log[prm->step] = id;
      prm->step += 1;
      prm->token = id;
      prm->pos += 1;
    }
  }
}

// Greedy over an arbitrary logits row (after the sampler rewrote logits in place).
__global__ void k_argmax_rows(const float* __restrict__ logits, int vocab, ArgmaxPart* __restrict__ part) {
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  float bv = -1e30f;
  int bi = kNoIndex;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    argmax_offer(bv, bi, logits[i], i);
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
    part[blockIdx.x] = ArgmaxPart{bv, bi};
  }
}

// ---------------------------------------------------------------------------------------------
// Isolated GEMV for 1..4 activation rows (the block-128 GEMV sweep): y[m][n] = W[n,:] . x[m,:].
// ---------------------------------------------------------------------------------------------
template <int MX, int R, int CPL>
__global__ void __launch_bounds__(kThreads) k_gemv(const float* __restrict__ x, QMat W, float* __restrict__ y) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const int K = W.K;
  float* bsum = xs + MX * K;
  for (int m = 0; m < MX; ++m) stage_copy(x + (size_t)m * K, xs + m * K, K);
  __syncthreads();
  for (int m = 0; m < MX; ++m) stage_block_sums(xs + m * K, bsum + m * (K / 128), K);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int g = blockIdx.x * kWarps + (threadIdx.x >> 5); g * R < W.N; g += gridDim.x * kWarps) {
    float out[MX][R];
    warp_gemv<MX, R, CPL>(W, g * R, xs, K, bsum, K / 128, out);
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MX; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) y[(size_t)m * W.N + g * R + r] = out[m][r];
    }
  }
}

}  // namespace le
