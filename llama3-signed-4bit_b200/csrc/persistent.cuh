// Persistent token-step kernel for batch-1 decode (sm_100a).
//
// One cooperative launch runs whole token steps (src/llama_engine.cpp:935-1042 and the greedy
// sampler :784-792): one CTA per SM, each with
//   * a producer warp that streams the CTA's weight records from HBM into a shared-memory ring
//     with cp.async.bulk (TMA bulk copies) and mbarriers, running ahead across phases and layers
//     (weights never depend on activations), and
//   * eight consumer warps that, phase by phase, wait for the phase's inputs through
//     release/acquire counters in global memory, stage the input vector as MMA digit fragments
//     (rms-norm fused where the reference normalises), and reduce their records on the integer
//     tensor-core path (mma_gemv.cuh).
// Phases of layer l: QKV rows -> attention per head (RoPE, KV append, softmax, PV) -> o-proj
// rows (+ residual) -> gate/up rows (SiLU * up) -> down rows (+ residual); then lm_head rows with
// a fused greedy argmax.  Every phase's work is split statically over the CTAs by a host-built
// schedule.  All waits are bounded in time; on timeout a global error word is set, every later
// wait returns immediately and the launch drains, so the host sees an error, never a hang.
//
// Record format (built at load time from the LLM4S128 matrices): 16 rows x 16 blocks
// (2048 columns) of one matrix, 17408 bytes:
//   [0, 16384): for block j = 0..15, lane L = 0..31 (g = L/4, t = L%4): 16 bytes of row g at
//               block bytes [16t, 16t+16), then 16 bytes of row g+8 (the MMA A fragments);
//   [16384, 17408): for block j, row r = 0..15: u32 = step_bf16 | min_bf16 << 16.
#pragma once

#include "mma_gemv.cuh"

namespace le {

constexpr int kRecBytes = 17408;
constexpr int kRecNibBytes = 16384;
constexpr int kPConsumerWarps = 8;
constexpr int kPThreads = 32 * (kPConsumerWarps + 1);
constexpr int kRingSlots = 10;
constexpr int kMiscFloats = 1536;  // attention scratch (q, k, v, reductions, 16x64 partials)
constexpr int kImageBytes = 32768 + 1024;  // digit fragments for K <= 8192, or attention scores
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s bound on every wait

enum PKind : uint16_t { PK_QKV = 0, PK_ATTN, PK_O, PK_GATEUP, PK_DOWN, PK_LMHEAD };

struct PItem {
  uint16_t kind, layer;
  uint32_t tile;      // row tile (16 rows) within the phase's row space; head index for PK_ATTN
  uint32_t rec;       // first record of the item in the CTA's per-token record stream
  uint16_t nrec, warp;
};

struct PSeg {
  uint16_t kind, layer;
  uint32_t item_begin, item_end;
};

struct PCtaSched {
  uint32_t seg_off, nseg;
  uint32_t item_off, nitem;
  uint32_t rec_off, nrec;  // records per token (all of them; the lm_head ones come last)
  uint32_t nrec_nolm;      // records per token without the lm_head
  uint32_t pad;
};

// Control words, zero-initialised at engine creation.
struct PCtrl {
  uint32_t step_seq;   // token steps completed by earlier launches
  uint32_t lm_seq;     // token steps with logits completed by earlier launches
  uint32_t done_ctas;  // CTAs finished in the current launch
  uint32_t error;      // nonzero after a wait timed out
  uint32_t err_where;  // code of the first wait that timed out
  uint32_t pad[3];
  unsigned long long key[3];  // packed greedy candidates, by lm step modulo 3
};

struct PArgs {
  const uint8_t* arena;           // repacked records
  const PCtaSched* sched;
  const PSeg* segs;
  const PItem* items;
  const unsigned long long* recs; // byte offsets of records in `arena`
  const float* const* norms;      // [2*layers + 1]: in_norm[l], post_norm[l] ..., final_norm
  const float* rope_cos;
  const float* rope_sin;
  float* x;         // [dim]
  float* qkv;       // [dim + 2*kv_dim]
  float* attn;      // [dim]
  float* act;       // [ffn]
  float* logits;    // [vocab]
  float* kcache;    // slot 0: [layers][max_seq][kv_dim]
  float* vcache;
  uint32_t* ctr;    // counters
  PCtrl* ctrl;
  const StepParams* prm;
  int32_t* token_log;
  int32_t* am_result;
  unsigned long long lm_rec_base;  // record offset of lm_head tile 0 (embedding lookup)
  int layers, dim, ffn, vocab, heads, kv_heads, max_seq;
  int n_qkv_items, n_o_items, n_gu_items, n_down_items, n_lm_ctas;
  int n_tokens, do_logits;
  unsigned long long* trace;  // optional: per CTA kTraceCap (time, tag) pairs, first token only
};

constexpr int kTraceCap = 1024;

// Counter layout: per layer 5 counters, then emb and lm.
__host__ __device__ inline int ctr_x(int l) { return 5 * l + 0; }   // x ready for layer l (l >= 1)
__host__ __device__ inline int ctr_qkv(int l) { return 5 * l + 1; }
__host__ __device__ inline int ctr_attn(int l) { return 5 * l + 2; }
__host__ __device__ inline int ctr_o(int l) { return 5 * l + 3; }
__host__ __device__ inline int ctr_act(int l) { return 5 * l + 4; }
__host__ __device__ inline int ctr_emb(int layers) { return 5 * layers + 5; }
__host__ __device__ inline int ctr_lm(int layers) { return 5 * layers + 6; }
__host__ __device__ inline int ctr_count(int layers) { return 5 * layers + 8; }

// ---------------------------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ void mbar_arrive_n(uint32_t a, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(n) : "memory");
}
__device__ __forceinline__ void group_sync(int group, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(2 + group), "r"(nthreads) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kPConsumerWarps) : "memory");
}
__device__ __forceinline__ bool reached(uint32_t v, uint32_t target) { return (int32_t)(v - target) >= 0; }

__device__ __forceinline__ bool failed(const PArgs& A) {
  return *reinterpret_cast<volatile uint32_t*>(&A.ctrl->error) != 0u;
}
__device__ __forceinline__ void fail(const PArgs& A, uint32_t where) {
  if (atomicCAS(&A.ctrl->error, 0u, 1u) == 0u) A.ctrl->err_where = where;
}

// Bounded wait for a global counter.  Returns false (and flags the launch) on timeout.
__device__ bool wait_counter(const PArgs& A, int c, uint32_t target, uint32_t where) {
  const uint32_t* p = A.ctr + c;
  if (reached(ld_acquire(p), target)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    if (failed(A)) return false;
    if (reached(ld_acquire(p), target)) return true;
    if (gtimer() - t0 > kWaitNs) { fail(A, where); return false; }
    __nanosleep(40);
  }
}

__device__ bool wait_mbar(const PArgs& A, uint32_t bar, uint32_t parity, uint32_t where) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (failed(A)) return false;
    if (gtimer() - t0 > kWaitNs) { fail(A, where); return false; }
  }
}

// Release of one unit of work: every lane fences its own stores, then lane 0 adds.
__device__ __forceinline__ void warp_signal(uint32_t* ctr) {
  __threadfence();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) atomicAdd(ctr, 1u);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(~(uint32_t)idx);
}

// ---------------------------------------------------------------------------------------------
// Staging: the consumer group (256 threads) turns an input vector into MX = 1 digit fragments
//   bfrag[(b*4 + i)*16 + p*4 + t] = (b0, b1) for digit plane p, MMA i, quad lane t of block b,
// plus block sums and scales.  Thread `tid` owns 8-element groups q = tid + 256*r; group q
// covers elements 8q..8q+7 = block q/16, (t, i) = ((q%16)/4, (q%16)%4).
// ---------------------------------------------------------------------------------------------
struct Stage {
  uint2* bfrag;
  float* bsum;
  float* escl;
  float* red;  // 16 floats
};

template <int G>  // groups of 8 per thread: 1 for K = 2048, 4 for K = 8192
__device__ __forceinline__ void stage_groups(float (&v)[G][8], int K, const Stage& S) {
  const int tid = threadIdx.x - 32;
#pragma unroll
  for (int r = 0; r < G; ++r) {
    const int q = tid + 256 * r;
    const int b = q >> 4, ti = q & 15, t = ti >> 2, i = ti & 3;
    float s = 0.0f, a = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      s += v[r][e];
      a = fmaxf(a, fabsf(v[r][e]));
    }
    // the 16 threads of a block are a half warp
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    }
    // a < 2^ex with ex from the exponent field (denormals bounded by 2^-126)
    const int ex = max((int)((__float_as_uint(a) >> 23) & 0xFFu), 1) - 126;
    const int e = min(29 - ex, 126);
    const float up = __uint_as_float((uint32_t)(e + 127) << 23);  // 2^e, exact scaling
    if (ti == 0) {
      S.bsum[b] = s;
      S.escl[b] = a > 0.0f ? __uint_as_float((uint32_t)(127 - e) << 23) : 0.0f;
    }
    uint32_t w[4][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      int X = __float2int_rn(v[r][k] * up);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int d = ((X + 128) & 255) - 128;
        X = (X - d) >> 8;
        w[p][k & 1] |= (uint32_t)(d & 255) << (8 * (k >> 1));
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) S.bfrag[(b * 4 + i) * 16 + p * 4 + t] = make_uint2(w[p][0], w[p][1]);
  }
  (void)K;
}

// rms-norm staging of a 2048-wide activation (one group per thread): out = x * g * inv.
// `x` was produced inside this launch, so it is read through L2 (ld.cg).  Writes the normalised
// values to `keep` (if non-null; used by nothing else than callers that need them).
__device__ __forceinline__ void stage_norm2048(const float* x, const float* gamma, const Stage& S) {
  const int tid = threadIdx.x - 32;
  float v[1][8];
  const float4 a = __ldcg(reinterpret_cast<const float4*>(x) + 2 * tid);
  const float4 b = __ldcg(reinterpret_cast<const float4*>(x) + 2 * tid + 1);
  const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * tid);
  const float4 gb = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * tid + 1);
  float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss = fmaf(xv[k], xv[k], ss);
  ss = warp_sum(ss);
  if ((tid & 31) == 0) S.red[tid >> 5] = ss;
  consumer_sync();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kPConsumerWarps; ++w) tot += S.red[w];
  const float inv = 1.0f / sqrtf(tot / 2048.0f + 1e-5f);
#pragma unroll
  for (int k = 0; k < 8; ++k) v[0][k] = __fmul_rn(__fmul_rn(xv[k], gv[k]), inv);
  stage_groups<1>(v, 2048, S);
  consumer_sync();
}

// plain staging of a 2048-wide (G=1) or 8192-wide (G=4) activation
template <int G>
__device__ __forceinline__ void stage_plain(const float* x, const Stage& S) {
  const int tid = threadIdx.x - 32;
  float v[G][8];
#pragma unroll
  for (int r = 0; r < G; ++r) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(x) + 2 * (tid + 256 * r));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(x) + 2 * (tid + 256 * r) + 1);
    v[r][0] = a.x; v[r][1] = a.y; v[r][2] = a.z; v[r][3] = a.w;
    v[r][4] = b.x; v[r][5] = b.y; v[r][6] = b.z; v[r][7] = b.w;
  }
  stage_groups<G>(v, 256 * G * 8, S);
  consumer_sync();
}

// ---------------------------------------------------------------------------------------------
// One record (16 rows x 16 blocks) on the MMA path, split over the consumer warps: warp cw
// reduces blocks 2*cw and 2*cw+1 (of kq*16 .. kq*16+15 of the staged input).  The four MMAs of a
// block use independent accumulators (their int32 sums are exact), so they issue back to back.
// Lanes with t == 0 return the partial sums of rows g (p0) and g+8 (p1).
// ---------------------------------------------------------------------------------------------
template <int NBLK>
__device__ __forceinline__ void record_part(const uint8_t* rec, int kq, int j0, const Stage& S, float& p0, float& p1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint4* nib = reinterpret_cast<const uint4*>(rec);
  const uint32_t* sc = reinterpret_cast<const uint32_t*>(rec + kRecNibBytes);
  p0 = 0.0f;
  p1 = 0.0f;
#pragma unroll 2
  for (int jj = 0; jj < NBLK; ++jj) {
    const int j = j0 + jj, b = kq * 16 + j;
    const uint4 wa = nib[j * 64 + lane * 2];
    const uint4 wb = nib[j * 64 + lane * 2 + 1];
    int c[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0;
      const uint32_t xa = i == 0 ? wa.x : i == 1 ? wa.y : i == 2 ? wa.z : wa.w;
      const uint32_t xb = i == 0 ? wb.x : i == 1 ? wb.y : i == 2 ? wb.z : wb.w;
      const uint2 bb = lane < 16 ? S.bfrag[(b * 4 + i) * 16 + lane] : make_uint2(0u, 0u);
      mma_u8s8(c[i], xa & 0x0F0F0F0Fu, xb & 0x0F0F0F0Fu, (xa >> 4) & 0x0F0F0F0Fu, (xb >> 4) & 0x0F0F0F0Fu, bb.x, bb.y);
    }
    int cs[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) cs[e] = (c[0][e] + c[1][e]) + (c[2][e] + c[3][e]);
    const int p2 = __shfl_xor_sync(0xffffffffu, cs[0], 1);
    const int p3 = __shfl_xor_sync(0xffffffffu, cs[1], 1);
    const int q2 = __shfl_xor_sync(0xffffffffu, cs[2], 1);
    const int q3 = __shfl_xor_sync(0xffffffffu, cs[3], 1);
    if (t == 0) {
      const uint32_t s0 = sc[j * 16 + g], s1 = sc[j * 16 + g + 8];
      const float es = S.escl[b], xsb = S.bsum[b];
      float v0 = (float)p3;
      v0 = fmaf(v0, 256.0f, (float)p2);
      v0 = fmaf(v0, 256.0f, (float)cs[1]);
      v0 = fmaf(v0, 256.0f, (float)cs[0]);
      float v1 = (float)q3;
      v1 = fmaf(v1, 256.0f, (float)q2);
      v1 = fmaf(v1, 256.0f, (float)cs[3]);
      v1 = fmaf(v1, 256.0f, (float)cs[2]);
      p0 += fmaf(bf16_bits_to_f32(s0 & 0xFFFFu) * es, v0, bf16_bits_to_f32(s0 >> 16) * xsb);
      p1 += fmaf(bf16_bits_to_f32(s1 & 0xFFFFu) * es, v1, bf16_bits_to_f32(s1 >> 16) * xsb);
    }
  }
}

__device__ __forceinline__ void record_blocks(int F, const uint8_t* rec, int kq, int mi, const Stage& S, float& p0,
                                              float& p1) {
  switch (F) {
    case 1: record_part<16>(rec, kq, 0, S, p0, p1); break;
    case 2: record_part<8>(rec, kq, 8 * mi, S, p0, p1); break;
    case 4: record_part<4>(rec, kq, 4 * mi, S, p0, p1); break;
    default: record_part<2>(rec, kq, 2 * mi, S, p0, p1); break;
  }
}

// ---------------------------------------------------------------------------------------------
// Attention of one head on the consumer group (src/llama_engine.cpp:953-1021).
// ---------------------------------------------------------------------------------------------
__device__ void attention_head(const PArgs& A, int l, int h, int pos, float* scores, float* sm) {
  const int tid = threadIdx.x - 32;
  const int group = A.heads / A.kv_heads, kvh = h / group;
  const int kv_dim = A.kv_heads * LE_HEAD_DIM, q_dim = A.heads * LE_HEAD_DIM;
  float* sq = sm;            // 64
  float* sk = sm + 64;       // 64
  float* sv = sm + 128;      // 64
  float* red = sm + 192;     // 16
  float* pv = sm + 256;      // 16 x 64 partial outputs (1024 floats)
  float* kc = A.kcache + (size_t)l * A.max_seq * kv_dim + kvh * LE_HEAD_DIM;
  float* vc = A.vcache + (size_t)l * A.max_seq * kv_dim + kvh * LE_HEAD_DIM;
  if (tid < 32) {
    const float c = A.rope_cos[pos * 32 + tid], s = A.rope_sin[pos * 32 + tid];
    const float r0 = __ldcg(A.qkv + h * LE_HEAD_DIM + tid), r1 = __ldcg(A.qkv + h * LE_HEAD_DIM + tid + 32);
    sq[tid] = __fsub_rn(__fmul_rn(r0, c), __fmul_rn(r1, s));
    sq[tid + 32] = __fadd_rn(__fmul_rn(r0, s), __fmul_rn(r1, c));
  } else if (tid < 64) {
    const int i = tid - 32;
    const float c = A.rope_cos[pos * 32 + i], s = A.rope_sin[pos * 32 + i];
    const float* kh = A.qkv + q_dim + kvh * LE_HEAD_DIM;
    const float r0 = __ldcg(kh + i), r1 = __ldcg(kh + i + 32);
    sk[i] = __fsub_rn(__fmul_rn(r0, c), __fmul_rn(r1, s));
    sk[i + 32] = __fadd_rn(__fmul_rn(r0, s), __fmul_rn(r1, c));
  } else if (tid < 128) {
    sv[tid - 64] = __ldcg(A.qkv + q_dim + kv_dim + kvh * LE_HEAD_DIM + tid - 64);
  }
  consumer_sync();
  if (h % group == 0 && tid < 64) {
    kc[(size_t)pos * kv_dim + tid] = sk[tid];
    vc[(size_t)pos * kv_dim + tid] = sv[tid];
  }
  // scores: one position per thread, the 16 row loads issued together
  float mx = -INFINITY;
  for (int t = tid; t <= pos; t += 256) {
    float dot = 0.0f;
    if (t == pos) {
#pragma unroll
      for (int d = 0; d < 64; ++d) dot = fmaf(sq[d], sk[d], dot);
    } else {
      const float4* kt = reinterpret_cast<const float4*>(kc + (size_t)t * kv_dim);
      float4 k4[16];
#pragma unroll
      for (int d4 = 0; d4 < 16; ++d4) k4[d4] = __ldcg(kt + d4);
#pragma unroll
      for (int d4 = 0; d4 < 16; ++d4) {
        dot = fmaf(sq[4 * d4], k4[d4].x, dot);
        dot = fmaf(sq[4 * d4 + 1], k4[d4].y, dot);
        dot = fmaf(sq[4 * d4 + 2], k4[d4].z, dot);
        dot = fmaf(sq[4 * d4 + 3], k4[d4].w, dot);
      }
    }
    const float s = dot * 0.125f;
    scores[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  consumer_sync();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kPConsumerWarps; ++w) mx = fmaxf(mx, red[w]);
  float se = 0.0f;
  for (int t = tid; t <= pos; t += 256) {
    const float e = expf(scores[t] - mx);
    scores[t] = e;
    se += e;
  }
  se = warp_sum(se);
  consumer_sync();  // everyone has read red[0..7] and written scores[]
  if ((tid & 31) == 0) red[8 + (tid >> 5)] = se;
  consumer_sync();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kPConsumerWarps; ++w) tot += red[8 + w];
  const float inv = 1.0f / tot;
  // PV: thread = (4 dims d4, position group tg of 16); loads unrolled by 4
  const int d4 = tid & 15, tg = tid >> 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 svn = reinterpret_cast<const float4*>(sv)[d4];
  int t = tg;
  for (; t + 48 < pos; t += 64) {  // rows < pos only: row pos may still be in flight
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcg(reinterpret_cast<const float4*>(vc + (size_t)(t + 16 * u) * kv_dim) + d4);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float p = scores[t + 16 * u] * inv;
      acc.x = fmaf(p, v[u].x, acc.x);
      acc.y = fmaf(p, v[u].y, acc.y);
      acc.z = fmaf(p, v[u].z, acc.z);
      acc.w = fmaf(p, v[u].w, acc.w);
    }
  }
  for (; t <= pos; t += 16) {
    const float4 v = t == pos ? svn : __ldcg(reinterpret_cast<const float4*>(vc + (size_t)t * kv_dim) + d4);
    const float p = scores[t] * inv;
    acc.x = fmaf(p, v.x, acc.x);
    acc.y = fmaf(p, v.y, acc.y);
    acc.z = fmaf(p, v.z, acc.z);
    acc.w = fmaf(p, v.w, acc.w);
  }
  reinterpret_cast<float4*>(pv)[tg * 16 + d4] = acc;
  consumer_sync();
  if (tid < 64) {
    float o = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) o += pv[k * 64 + tid];
    A.attn[h * LE_HEAD_DIM + tid] = o;
    __threadfence();
  }
  consumer_sync();
  if (tid == 0) atomicAdd(A.ctr + ctr_attn(l), 1u);
}

// Embedding row `token` of the tied lm_head, read from its records, as 8 values per thread
// (elements 8*tid .. 8*tid+7 of the 2048-wide row; dequantize_embedding_row, :182-220).
__device__ __forceinline__ void embed_group(const PArgs& A, int token, float (&v)[8]) {
  const int tid = threadIdx.x - 32;
  const int T = token >> 4, gr = token & 15;
  const uint8_t* rec = A.arena + A.lm_rec_base + (unsigned long long)T * kRecBytes;
  const int b = tid >> 4, q = tid & 15, t = q >> 2, i = q & 3;
  const int L = (gr & 7) * 4 + t, half = gr >> 3;
  const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(rec + b * 1024 + L * 32 + half * 16 + 4 * i));
  const uint32_t s = __ldg(reinterpret_cast<const uint32_t*>(rec + kRecNibBytes + b * 64 + gr * 4));
  const float st = bf16_bits_to_f32(s & 0xFFFFu), mv = bf16_bits_to_f32(s >> 16);
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = __fadd_rn(mv, __fmul_rn((float)((w >> (4 * k)) & 0xFu), st));
}

// ---------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void trace_mark(const PArgs& A, int& n, int tok, uint32_t tag) {
  if (A.trace != nullptr && tok == 0 && n < kTraceCap) {
    unsigned long long* tr = A.trace + ((size_t)blockIdx.x * kTraceCap + n) * 2;
    tr[0] = gtimer();
    tr[1] = tag;
    ++n;
  }
}

__global__ void __launch_bounds__(kPThreads, 1) k_decode_persistent(const __grid_constant__ PArgs A) {
  extern __shared__ __align__(1024) uint8_t psmem[];
  uint8_t* ring = psmem;                                          // kRingSlots * kRecBytes
  uint8_t* image = ring + (size_t)kRingSlots * kRecBytes;          // kImageBytes
  float* misc = reinterpret_cast<float*>(image + kImageBytes);     // kMiscFloats
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(misc + kMiscFloats);  // 2*kRingSlots
  __shared__ float s_part[2][kPConsumerWarps][16];
  __shared__ unsigned long long s_best[kPConsumerWarps];
  __shared__ int s_token;

  const PCtaSched cs = A.sched[blockIdx.x];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kRingSlots);
  const uint32_t step_seq = A.ctrl->step_seq, lm_seq = A.ctrl->lm_seq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRingSlots; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kPConsumerWarps);  // arrivals are weighted: 8 per consumed record
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint32_t per_tok = A.do_logits ? cs.nrec : cs.nrec_nolm;
      const uint32_t total = per_tok * (uint32_t)A.n_tokens;
      uint32_t issued = 0;
      for (uint32_t q = 0; q < total; ++q) {
        const uint32_t slot = q % kRingSlots, use = q / kRingSlots;
        if (use > 0 && !wait_mbar(A, empty0 + 8 * slot, (use - 1) & 1, 1)) break;
        const uint32_t r = q % per_tok;
        const unsigned long long off = A.recs[cs.rec_off + r];
        mbar_expect_tx(full0 + 8 * slot, kRecBytes);
        bulk_g2s(smem_u32(ring + (size_t)slot * kRecBytes), A.arena + off, kRecBytes, full0 + 8 * slot);
        issued = q + 1;
      }
      // drain: never leave bulk copies in flight into a CTA that is about to exit
      for (uint32_t q = (issued > kRingSlots ? issued - kRingSlots : 0); q < issued; ++q)
        wait_mbar(A, full0 + 8 * (q % kRingSlots), (q / kRingSlots) & 1, 2);
    }
  } else {
    // ---------------- consumers ----------------
    const int cw = warp - 1;  // consumer warp index
    const int tid = threadIdx.x - 32;
    Stage S;
    S.bfrag = reinterpret_cast<uint2*>(image);
    S.bsum = reinterpret_cast<float*>(image + 32768);
    S.escl = S.bsum + 64;
    S.red = S.escl + 64;
    float* scores = reinterpret_cast<float*>(image);  // attention reuses the image buffer
    const uint32_t per_tok = A.do_logits ? cs.nrec : cs.nrec_nolm;
    int token = A.prm->token;
    const int pos0 = A.prm->pos;
    int ntr = 0;
    int buf = 0;

    for (int tok = 0; tok < A.n_tokens; ++tok) {
      const uint32_t s = step_seq + (uint32_t)tok;
      const int pos = pos0 + tok;
      const uint32_t rec_base = per_tok * (uint32_t)tok;
      if (tid == 0) trace_mark(A, ntr, tok, 0xFFFF0000u);
      if (tok > 0) {
        // next token = greedy id of the previous step (all CTAs' lm_head work done)
        if (tid == 0) {
          wait_counter(A, ctr_lm(A.layers), (lm_seq + (uint32_t)tok) * (uint32_t)A.n_lm_ctas, 3);
          const unsigned long long k = atomicAdd(&A.ctrl->key[(lm_seq + tok - 1) % 3], 0ull);
          s_token = k == 0ull ? 0 : (int)(~(uint32_t)(k & 0xFFFFFFFFull));
        }
        consumer_sync();
        token = s_token;
      }
      // CTA 0: embedding into x, token log, reset of the next greedy key
      float emb[8];
      embed_group(A, token, emb);
      if (blockIdx.x == 0) {
        float4* xo = reinterpret_cast<float4*>(A.x) + 2 * tid;
        xo[0] = make_float4(emb[0], emb[1], emb[2], emb[3]);
        xo[1] = make_float4(emb[4], emb[5], emb[6], emb[7]);
        if (tid == 0) {
          A.ctrl->key[(lm_seq + tok + 1) % 3] = 0ull;
          if (tok > 0) A.token_log[tok - 1] = token;
        }
        __threadfence();
        consumer_sync();
        if (tid == 0) atomicAdd(A.ctr + ctr_emb(A.layers), 1u);
      }

      for (uint32_t si = 0; si < cs.nseg; ++si) {
        const PSeg sg = A.segs[cs.seg_off + si];
        const int l = sg.layer;
        if (sg.kind == PK_LMHEAD && !A.do_logits) continue;
        const uint32_t tag = ((uint32_t)sg.kind << 8) | (uint32_t)l;
        if (tid == 0) trace_mark(A, ntr, tok, tag | 0x10000u);
        // ---- dependency + staging ----
        switch (sg.kind) {
          case PK_QKV: {
            if (l == 0) {
              // the input is the embedding computed above (no wait)
              const float* gm = A.norms[0];
              float ss = 0.0f;
#pragma unroll
              for (int k = 0; k < 8; ++k) ss = fmaf(emb[k], emb[k], ss);
              ss = warp_sum(ss);
              if (lane == 0) S.red[cw] = ss;
              consumer_sync();
              if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
              float tot = 0.0f;
#pragma unroll
              for (int w = 0; w < kPConsumerWarps; ++w) tot += S.red[w];
              const float inv = 1.0f / sqrtf(tot / 2048.0f + 1e-5f);
              const float4 ga = __ldg(reinterpret_cast<const float4*>(gm) + 2 * tid);
              const float4 gb = __ldg(reinterpret_cast<const float4*>(gm) + 2 * tid + 1);
              const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
              float v[1][8];
#pragma unroll
              for (int k = 0; k < 8; ++k) v[0][k] = __fmul_rn(__fmul_rn(emb[k], gv[k]), inv);
              stage_groups<1>(v, 2048, S);
              consumer_sync();
            } else {
              if (tid == 0) wait_counter(A, ctr_x(l), (s + 1) * (uint32_t)A.n_down_items, 10 + l);
              consumer_sync();
              if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
              stage_norm2048(A.x, A.norms[2 * l], S);
            }
            break;
          }
          case PK_ATTN:
            if (tid == 0) wait_counter(A, ctr_qkv(l), (s + 1) * (uint32_t)A.n_qkv_items, 100 + l);
            consumer_sync();
            if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
            break;
          case PK_O:
            if (tid == 0) {
              wait_counter(A, ctr_attn(l), (s + 1) * (uint32_t)A.heads, 200 + l);
              if (l == 0) wait_counter(A, ctr_emb(A.layers), s + 1, 290);
            }
            consumer_sync();
            if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
            stage_plain<1>(A.attn, S);
            break;
          case PK_GATEUP:
            if (tid == 0) wait_counter(A, ctr_o(l), (s + 1) * (uint32_t)A.n_o_items, 300 + l);
            consumer_sync();
            if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
            stage_norm2048(A.x, A.norms[2 * l + 1], S);
            break;
          case PK_DOWN:
            if (tid == 0) wait_counter(A, ctr_act(l), (s + 1) * (uint32_t)A.n_gu_items, 400 + l);
            consumer_sync();
            if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
            if (A.ffn == 8192) stage_plain<4>(A.act, S);
            else if (A.ffn == 4096) stage_plain<2>(A.act, S);
            else stage_plain<1>(A.act, S);
            break;
          case PK_LMHEAD:
            if (tid == 0) wait_counter(A, ctr_x(A.layers), (s + 1) * (uint32_t)A.n_down_items, 500);
            consumer_sync();
            if (tid == 0) trace_mark(A, ntr, tok, tag | 0x20000u);
            stage_norm2048(A.x, A.norms[2 * A.layers], S);
            break;
        }
        if (tid == 0) trace_mark(A, ntr, tok, tag | 0x30000u);
        // ---- work ----
        if (sg.kind == PK_ATTN) {
          for (uint32_t it = sg.item_begin; it < sg.item_end; ++it) {
            attention_head(A, l, (int)A.items[cs.item_off + it].tile, pos, scores, misc);
            consumer_sync();
          }
          if (tid == 0) trace_mark(A, ntr, tok, tag | 0x40000u);
          continue;
        }
        // Split factor F: groups of F warps share one item, each warp reducing 16/F blocks of every
        // record of it; F = 1 (one warp per item) when the CTA has at least 8 items in the phase.
        const int n_items = (int)(sg.item_end - sg.item_begin);
        const int F = n_items >= 8 ? 1 : n_items >= 4 ? 2 : n_items >= 2 ? 4 : 8;
        const int n_groups = kPConsumerWarps / F, gi = cw / F, mi = cw % F;
        unsigned long long best = 0ull;
        unsigned long long wait_cycles = 0;
        for (int ii = gi; ii < n_items; ii += n_groups) {
          const PItem item = A.items[cs.item_off + sg.item_begin + ii];
          float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [record kind: gate/up][row g, g+8]
          for (int rr = 0; rr < item.nrec; ++rr) {
            const uint32_t q = rec_base + item.rec + rr;
            const uint32_t slot = q % kRingSlots;
            const long long w0 = clock64();
            wait_mbar(A, full0 + 8 * slot, (q / kRingSlots) & 1, 600 + item.kind);
            wait_cycles += (unsigned long long)(clock64() - w0);
            float p0, p1;
            record_blocks(F, ring + (size_t)slot * kRecBytes, item.kind == PK_DOWN ? rr : 0, mi, S, p0, p1);
            __syncwarp();
            if (lane == 0) mbar_arrive_n(empty0 + 8 * slot, (uint32_t)(kPConsumerWarps / F));
            const int k = item.kind == PK_GATEUP ? rr : 0;
            if (F == 1) {
              acc[k][0] += p0;
              acc[k][1] += p1;
            } else {
              if ((lane & 3) == 0) {
                s_part[buf][cw][lane >> 2] = p0;
                s_part[buf][cw][(lane >> 2) + 8] = p1;
              }
              group_sync(gi, 32 * F);
              if (mi == 0 && (lane & 3) == 0) {
                float v0 = 0.f, v1 = 0.f;
                for (int w = 0; w < F; ++w) {
                  v0 += s_part[buf][gi * F + w][lane >> 2];
                  v1 += s_part[buf][gi * F + w][(lane >> 2) + 8];
                }
                acc[k][0] += v0;
                acc[k][1] += v1;
              }
              buf ^= 1;
            }
          }
          // epilogue: lanes t == 0 of the group's first warp own rows g and g+8
          if (mi == 0 && (lane & 3) == 0) {
            const int r0 = (int)item.tile * 16 + (lane >> 2), r1 = r0 + 8;
            switch (item.kind) {
              case PK_QKV:
                A.qkv[r0] = acc[0][0];
                A.qkv[r1] = acc[0][1];
                break;
              case PK_O:
              case PK_DOWN:
                A.x[r0] = __ldcg(A.x + r0) + acc[0][0];
                A.x[r1] = __ldcg(A.x + r1) + acc[0][1];
                break;
              case PK_GATEUP:
                A.act[r0] = (acc[0][0] / (1.0f + expf(-acc[0][0]))) * acc[1][0];
                A.act[r1] = (acc[0][1] / (1.0f + expf(-acc[0][1]))) * acc[1][1];
                break;
              case PK_LMHEAD:
                A.logits[r0] = acc[0][0];
                A.logits[r1] = acc[0][1];
                if (acc[0][0] > -1e30f) best = max(best, argmax_key(acc[0][0], r0));
                if (acc[0][1] > -1e30f) best = max(best, argmax_key(acc[0][1], r1));
                break;
            }
            __threadfence();
          }
          if (mi == 0) {
            __syncwarp();
            if (lane == 0 && item.kind != PK_LMHEAD) {
              uint32_t* c = A.ctr + (item.kind == PK_QKV ? ctr_qkv(l)
                                     : item.kind == PK_O  ? ctr_o(l)
                                     : item.kind == PK_GATEUP ? ctr_act(l)
                                                              : ctr_x(l + 1));
              atomicAdd(c, 1u);
            }
          }
        }
        if (sg.kind == PK_LMHEAD) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
          if (lane == 0) s_best[cw] = best;
          consumer_sync();
          if (tid == 0) {
            for (int w = 0; w < kPConsumerWarps; ++w) best = max(best, s_best[w]);
            atomicMax(&A.ctrl->key[(lm_seq + tok) % 3], best);
            __threadfence();
            atomicAdd(A.ctr + ctr_lm(A.layers), 1u);
          }
        }
        if (cw == 0 && lane == 0 && A.trace != nullptr && tok == 0 && ntr < kTraceCap) {
          unsigned long long* tr = A.trace + ((size_t)blockIdx.x * kTraceCap + ntr) * 2;
          tr[0] = wait_cycles;
          tr[1] = tag | 0x50000u;
          ++ntr;
        }
        if (tid == 0) trace_mark(A, ntr, tok, tag | 0x40000u);
      }
    }
  }

  // ---------------- launch epilogue ----------------
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&A.ctrl->done_ctas, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      if (A.do_logits) {
        const int last = A.n_tokens - 1;
        const unsigned long long k = atomicAdd(&A.ctrl->key[(lm_seq + last) % 3], 0ull);
        const int id = k == 0ull ? 0 : (int)(~(uint32_t)(k & 0xFFFFFFFFull));
        A.am_result[0] = id;
        if (A.n_tokens > 1) A.token_log[last] = id;
      }
      A.ctrl->step_seq = step_seq + (uint32_t)A.n_tokens;
      A.ctrl->lm_seq = lm_seq + (A.do_logits ? (uint32_t)A.n_tokens : 0u);
      A.ctrl->done_ctas = 0;
      __threadfence();
    }
  }
}

}  // namespace le

namespace le {

// Repack one LLM4S128 matrix (rows N % 16 == 0, K % 2048 == 0) into records
// (T, kq) -> dst + (T * K/2048 + kq) * kRecBytes.  One thread per 16-byte piece.
__global__ void k_repack(QMat W, uint8_t* __restrict__ dst) {
  const int KQ = W.K / 2048, nb = W.K / 128;
  const long long pieces_nib = (long long)W.N * (W.K / 32);       // 16-byte nibble pieces
  const long long pieces_sc = (long long)W.N * nb / 4;           // 4 scale words per piece
  const long long total = pieces_nib + pieces_sc;
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < total; p += (long long)gridDim.x * blockDim.x) {
    if (p < pieces_nib) {
      // source piece: row n, chunk c (16 bytes) of the row
      const int n = (int)(p / (W.K / 32)), c = (int)(p % (W.K / 32));
      const int b = c >> 2, t = c & 3;
      const int T = n >> 4, r = n & 15, g = r & 7, half = r >> 3;
      const int kq = b / 16, j = b % 16;
      const int L = g * 4 + t;
      uint8_t* rec = dst + ((size_t)T * KQ + kq) * kRecBytes;
      const uint4 v = *reinterpret_cast<const uint4*>(W.nib + (size_t)n * (W.K / 2) + (size_t)c * 16);
      *reinterpret_cast<uint4*>(rec + j * 1024 + L * 32 + half * 16) = v;
    } else {
      const long long q = p - pieces_nib;  // 4 consecutive (n, b) scale entries of one row
      const long long e0 = q * 4;
      const int n = (int)(e0 / nb), b0 = (int)(e0 % nb);
      const int T = n >> 4, r = n & 15;
      for (int e = 0; e < 4; ++e) {
        const int b = b0 + e, kq = b / 16, j = b % 16;
        uint8_t* rec = dst + ((size_t)T * KQ + kq) * kRecBytes;
        const size_t si = (size_t)n * nb + b;
        const uint32_t w = (uint32_t)W.step[si] | ((uint32_t)W.mn[si] << 16);
        *reinterpret_cast<uint32_t*>(rec + kRecNibBytes + (j * 16 + r) * 4) = w;
      }
    }
  }
}

}  // namespace le
