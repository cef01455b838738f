// Causal prefill attention on the tcgen05 tensor cores (sm_100a): the reference's per-head
// attention (src/llama_engine.cpp:958-1021: s_t = (q . k_t) * 0.125 for t <= pos, softmax,
// o = sum_t p_t v_t) for a prefill chunk of one sequence, every query of the chunk at once.
//
// One CTA of 4 warps per (kv head g, tile of 32 queries).  Its MMA rows are the 4 q heads of
// the kv head times the 32 queries (row 32 w + i: head 4 g + w, query i), M = 128; thread
// 32 w + i owns row 32 w + i, which is also tensor-memory lane 32 w + i, so the softmax of a
// row needs no exchange between threads.  Keys come in tiles of 64.  Per tile:
//   * the 128 threads load the tile's K rows and V rows (fp32, from the KV cache) and write them
//     as bf16 hi / lo parts (x = hi + lo) into shared memory in the UMMA K-major 128-byte
//     swizzled layout: K as [key][dim], V transposed as [dim][key];
//   * thread 0 issues S = Q K^T (tcgen05.mma kind::f16, M = 128, N = 64, A = Q and B = K from
//     shared memory, fp32 accumulator in tensor memory) as three products per 16-wide k step,
//     Q_hi K_hi + Q_hi K_lo + Q_lo K_hi (the lo x lo term is below fp32 rounding), and commits
//     to an mbarrier;
//   * each thread reads its row of S (tcgen05.ld), applies the 0.125 scale and the causal mask
//     (key position <= query position), updates its running max and sum (online softmax) and
//     writes the row's probabilities as bf16 hi / lo into shared memory (the A operand of the
//     next product);
//   * thread 0 issues O_tile = P V (A = P, B = V^T, N = 64 dims) in the same three products;
//     each thread adds its row of O_tile to its register accumulator after rescaling that by
//     exp(old max - new max).
// Q is loaded once per CTA (hi / lo, same layout).  The latest query tiles, which see the most
// keys, are dispatched first.  The online softmax rounds differently from the reference's
// max-then-exp-then-normalise loop; the parity tolerance (logits 1e-3 relative) covers it.
//
// All mbarrier waits are bounded; on timeout the kernel records an error word (the batched
// path's GEMM error word) and finishes without further waits on the tensor pipe.
#pragma once

#include "batch_kernels.cuh"
#include "tc_gemm.cuh"

namespace le {
namespace attn {

constexpr int kQ = 32;                   // queries per CTA (per q head)
constexpr int kKeys = 64;                // keys per tile
constexpr int kRows = 128;               // MMA rows: 4 q heads x 32 queries
constexpr int kRowBytes = 128;           // one K-major row: 64 bf16
constexpr int kQBytes = kRows * kRowBytes;   // Q hi (or lo): 16 KB
constexpr int kKBytes = kKeys * kRowBytes;   // K tile hi (or lo): 8 KB
constexpr int kVBytes = 64 * kRowBytes;      // V^T tile hi (or lo): 64 dims x 64 keys
constexpr int kPBytes = kRows * kRowBytes;   // P hi (or lo)
constexpr int kOffQ = 0;                 // Q hi, Q lo
constexpr int kOffK = kOffQ + 2 * kQBytes;   // K hi, K lo
constexpr int kOffV = kOffK + 2 * kKBytes;   // V^T hi, V^T lo
constexpr int kOffP = kOffV + 2 * kVBytes;   // P hi, P lo
constexpr int kSmemBytes = kOffP + 2 * kPBytes + 1024;  // + room to align the base to 1024
constexpr uint32_t kTmemCols = 128;      // S in columns 0..63, O_tile in 64..127

// Byte offset of 16-byte chunk c of row r in a K-major 128-byte-swizzled region.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * kRowBytes + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate), cta_group::1.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Three products A_hi B_hi + A_hi B_lo + A_lo B_hi over K = 64 (4 steps of 16) into d_tmem.
__device__ __forceinline__ void mma_hilo(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                         uint32_t idesc) {
  const uint32_t as[3] = {a_hi, a_hi, a_lo}, bs[3] = {b_hi, b_lo, b_hi};
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    const uint64_t ad = tc::sw128_desc(as[p]), bd = tc::sw128_desc(bs[p]);
#pragma unroll
    for (int k = 0; k < 4; ++k)  // a 16-wide k step is 32 bytes further along the 128-byte row
      mma_ss(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (p > 0 || k > 0) ? 1u : 0u);
  }
}

// Bounded wait for MMA completion phase `parity`; false (and the error word set) on timeout.
__device__ __forceinline__ bool wait_mma(uint32_t bar, uint32_t parity, uint32_t* error, unsigned long long wait_ns,
                                         volatile uint32_t* abort_flag) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (!mbar_try(bar, parity)) {
    if (*abort_flag) return false;
    if (gtimer() - t0 > wait_ns) {
      *abort_flag = 1u;
      atomicCAS(error, 0u, 20u);
      return false;
    }
  }
  return true;
}

}  // namespace attn

// q: rotated queries [T][q_dim] (rows of the chunk); kc / vc: the slot's K / V cache of this
// layer ([pos][kv_dim]), already holding the chunk's own keys; out: [T][q_dim].
// Grid (kv_heads, ceil(T / 32)), 128 threads, attn::kSmemBytes of dynamic shared memory.
__global__ void __launch_bounds__(128) k_attn_prefill_tc5(const float* __restrict__ q, int q_dim,
                                                          const float* __restrict__ kc, const float* __restrict__ vc,
                                                          int kv_dim, int p0, int T, float* __restrict__ out,
                                                          uint32_t* error, unsigned long long wait_ns) {
  using namespace attn;
  extern __shared__ uint8_t attn_smem_raw[];
  __shared__ __align__(8) unsigned long long s_bar;
  __shared__ uint32_t s_tmem;
  __shared__ volatile uint32_t s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.x;
  const int tok0 = (gridDim.y - 1 - blockIdx.y) * kQ;  // latest query tiles first
  const int h = 4 * g + warp;                           // this thread's q head
  const int qi = min(tok0 + lane, T - 1);               // its query (rows past T are not stored)
  const int qpos = p0 + qi;
  const int p_last = p0 + min(tok0 + kQ - 1, T - 1);
  const int ntiles = p_last / kKeys + 1;
  const uint32_t base = (smem_u32(attn_smem_raw) + 1023u) & ~1023u;
  const uint32_t bar = smem_u32(&s_bar);
  const uint32_t row = (uint32_t)tid;  // MMA row / tensor-memory lane of this thread

  grid_dep_launch();
  if (tid == 0) {
    s_abort = 0u;
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&s_tmem), kTmemCols);
    tc::tmem_relinquish();
  }
  grid_dep_wait();  // q and the cache rows come from the previous kernels of the step

  // Q: this thread's row (head h, query qi), 64 dims as hi / lo
  {
    const float* qr = q + (size_t)qi * q_dim + (size_t)h * LE_HEAD_DIM;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 a = *reinterpret_cast<const float4*>(qr + 8 * c);
      const float4 b = *reinterpret_cast<const float4*>(qr + 8 * c + 4);
      uint32_t hi[4], lo[4];
      split_bf16(a.x, a.y, hi[0], lo[0]);
      split_bf16(a.z, a.w, hi[1], lo[1]);
      split_bf16(b.x, b.y, hi[2], lo[2]);
      split_bf16(b.z, b.w, hi[3], lo[3]);
      attn::sts128(base + kOffQ + swz(row, c), hi[0], hi[1], hi[2], hi[3]);
      attn::sts128(base + kOffQ + kQBytes + swz(row, c), lo[0], lo[1], lo[2], lo[3]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t t_s = tmem + ((uint32_t)(32 * warp) << 16);  // this warp's lanes, column 0
  const uint32_t t_o = t_s + 64;
  const uint32_t idesc = tc::idesc_bf16(64);

  const float* Kb = kc + (size_t)g * LE_HEAD_DIM;
  const float* Vb = vc + (size_t)g * LE_HEAD_DIM;
  float o[LE_HEAD_DIM];
#pragma unroll
  for (int d = 0; d < LE_HEAD_DIM; ++d) o[d] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  uint32_t parity = 0;
  int n_commit = 0;  // thread 0: commits issued

  for (int kt = 0; kt < ntiles; ++kt) {
    const int k0 = kt * kKeys;
    // ---- K tile [key][dim] and V^T tile [dim][key] as bf16 hi / lo (keys past p_last read
    // row p_last: finite values that the causal mask removes) ----
    {
      const int key = tid >> 1, half = tid & 1;
      const float* kr = Kb + (size_t)min(k0 + key, p_last) * kv_dim + 32 * half;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = *reinterpret_cast<const float4*>(kr + 8 * i);
        const float4 b = *reinterpret_cast<const float4*>(kr + 8 * i + 4);
        uint32_t hi[4], lo[4];
        split_bf16(a.x, a.y, hi[0], lo[0]);
        split_bf16(a.z, a.w, hi[1], lo[1]);
        split_bf16(b.x, b.y, hi[2], lo[2]);
        split_bf16(b.z, b.w, hi[3], lo[3]);
        const int c = 4 * half + i;
        attn::sts128(base + kOffK + swz(key, c), hi[0], hi[1], hi[2], hi[3]);
        attn::sts128(base + kOffK + kKBytes + swz(key, c), lo[0], lo[1], lo[2], lo[3]);
      }
      const int d = tid >> 1;  // V^T row: dimension d, keys 32 half .. 32 half + 31
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = Vb[(size_t)min(k0 + 32 * half + 8 * i + e, p_last) * kv_dim + d];
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) split_bf16(v[2 * e], v[2 * e + 1], hi[e], lo[e]);
        const int c = 4 * half + i;
        attn::sts128(base + kOffV + swz(d, c), hi[0], hi[1], hi[2], hi[3]);
        attn::sts128(base + kOffV + kVBytes + swz(d, c), lo[0], lo[1], lo[2], lo[3]);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
    __syncthreads();
    // ---- S = Q K^T ----
    if (tid == 0 && !s_abort) {
      tc::tc_fence_after();
      attn::mma_hilo(tmem, base + kOffQ, base + kOffQ + kQBytes, base + kOffK, base + kOffK + kKBytes, idesc);
      tc::tc_commit(bar);
      ++n_commit;
    }
    attn::wait_mma(bar, parity, error, wait_ns, &s_abort);
    parity ^= 1u;
    tc::tc_fence_after();
    // ---- online softmax of this thread's row ----
    float s[kKeys];
    {
      uint32_t r0[32], r1[32];
      tc::tmem_ld32(t_s, r0);
      tc::tmem_ld32(t_s + 32, r1);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        s[j] = __uint_as_float(r0[j]);
        s[32 + j] = __uint_as_float(r1[j]);
      }
    }
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      s[j] = k0 + j <= qpos ? s[j] * 0.125f : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    const float mn = fmaxf(m, mt);  // tile 0 holds key 0 <= every query: finite from there on
    const float alpha = expf(m - mn);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      s[j] = expf(s[j] - mn);
      sum += s[j];
    }
    l = l * alpha + sum;
    m = mn;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) split_bf16(s[8 * c + 2 * e], s[8 * c + 2 * e + 1], hi[e], lo[e]);
      attn::sts128(base + kOffP + swz(row, c), hi[0], hi[1], hi[2], hi[3]);
      attn::sts128(base + kOffP + kPBytes + swz(row, c), lo[0], lo[1], lo[2], lo[3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::tc_fence_before();
    __syncthreads();
    // ---- O_tile = P V ----
    if (tid == 0 && !s_abort) {
      tc::tc_fence_after();
      attn::mma_hilo(tmem + 64, base + kOffP, base + kOffP + kPBytes, base + kOffV, base + kOffV + kVBytes, idesc);
      tc::tc_commit(bar);
      ++n_commit;
    }
    attn::wait_mma(bar, parity, error, wait_ns, &s_abort);
    parity ^= 1u;
    tc::tc_fence_after();
    {
      uint32_t r0[32], r1[32];
      tc::tmem_ld32(t_o, r0);
      tc::tmem_ld32(t_o + 32, r1);
      tc::tmem_wait_ld();
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        o[d] = fmaf(o[d], alpha, __uint_as_float(r0[d]));
        o[32 + d] = fmaf(o[32 + d], alpha, __uint_as_float(r1[d]));
      }
    }
    tc::tc_fence_before();
    __syncthreads();  // S / O_tile read and the shared tiles free before the next tile
  }
  if (tok0 + lane < T) {
    const float inv = 1.0f / l;
    float* orow = out + (size_t)(tok0 + lane) * q_dim + (size_t)h * LE_HEAD_DIM;
#pragma unroll
    for (int d = 0; d < LE_HEAD_DIM; d += 4)
      *reinterpret_cast<float4*>(orow + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
  }
  // every issued MMA has completed (each commit was waited for, or a wait gave up: then the
  // issuing thread waits once more, bounded, for its last commit before the tensor memory is
  // released)
  if (s_abort && tid == 0 && n_commit > 0) {
    const unsigned long long t0 = gtimer();
    while (!mbar_try(bar, (uint32_t)(n_commit - 1) & 1u) && gtimer() - t0 < wait_ns) {
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace le
