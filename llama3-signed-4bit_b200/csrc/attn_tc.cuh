// Causal prefill attention on the tcgen05 tensor cores (sm_100a): the reference's per-head
// attention (src/llama_engine.cpp:958-1021: s_t = (q . k_t) * 0.125 for t <= pos, softmax,
// o = sum_t p_t v_t) for a prefill chunk of one sequence, every query of the chunk at once.
//
// Two kernels per layer:
//   * k_kv_tiles turns the layer's K / V cache rows 0..p_last (fp32) into per-(kv head, 64-key
//     tile) images of 32 KB, laid out exactly as the attention kernel's shared memory wants them:
//     K as [key][dim] and V transposed as [dim][key], each as bf16 hi and lo parts (x = hi + lo)
//     in the UMMA K-major 128-byte-swizzled layout.  Keys past p_last are zeros.  Every key of
//     the sequence is converted once per chunk instead of once per query tile.
//   * k_attn_prefill_tc5: one CTA of 4 warps per (kv head g, tile of 32 queries).  Its MMA rows
//     are the 4 q heads of the kv head times the 32 queries (row 32 w + i: head 4 g + w, query i),
//     M = 128; thread 32 w + i owns row 32 w + i, which is also tensor-memory lane 32 w + i, so
//     the softmax of a row needs no exchange between threads.  Per 64-key tile j:
//       - thread 0 brings the tile image into one of two shared-memory stages with one bulk copy
//         (issued two tiles ahead, completion on the stage's mbarrier);
//       - thread 0 issues S_j = Q K_j^T (tcgen05.mma kind::f16, M = 128, N = 64, A = Q and B = K
//         from shared memory, fp32 accumulator in one of two tensor-memory S buffers) as three
//         products per 16-wide k step, Q_hi K_hi + Q_hi K_lo + Q_lo K_hi (the lo x lo term is
//         below fp32 rounding);
//       - each thread reads its row of S (tcgen05.ld), scales it to log2 units, applies the
//         causal mask (only on tiles that reach past the CTA's first query), updates its running
//         max and sum (online softmax, exp2) and writes the row's probabilities as bf16 hi / lo
//         back over S in tensor memory (tcgen05.st);
//       - thread 0 issues O_tile = P V_j (A = P from tensor memory, B = V^T from shared memory,
//         N = 64 dims, the same three products), then S_{j+1} into the other S buffer, so the
//         next score product runs while the threads fold O_tile into their register accumulator
//         (rescaled by 2^(old max - new max)).
// Q is loaded once per CTA (hi / lo, same layout).  The latest query tiles, which see the most
// keys, are dispatched first.  The online softmax rounds differently from the reference's
// max-then-exp-then-normalise loop; the parity tolerance (logits 1e-3 relative) covers it.
//
// All mbarrier waits are bounded; on timeout the kernel records an error word (the batched
// path's GEMM error word) and finishes without further work on the tensor pipe, after waiting
// (bounded) for its own MMAs and bulk copies in flight.
#pragma once

#include "batch_kernels.cuh"
#include "tc_gemm.cuh"

namespace le {
namespace attn {

constexpr int kQ = 32;                        // queries per CTA (per q head)
constexpr int kKeys = 64;                     // keys per tile
constexpr int kRows = 128;                    // MMA rows: 4 q heads x 32 queries
constexpr int kRowBytes = 128;                // one K-major row: 64 bf16
constexpr int kQBytes = kRows * kRowBytes;    // Q hi (or lo): 16 KB
constexpr int kPartBytes = 64 * kRowBytes;    // one part of a tile image: 8 KB
constexpr int kTileBytes = 4 * kPartBytes;    // K hi, K lo, V^T hi, V^T lo: 32 KB
constexpr int kStages = 2;
constexpr int kOffQ = 0;                      // Q hi, Q lo
constexpr int kOffStage = 2 * kQBytes;        // stage s at kOffStage + s * kTileBytes
constexpr int kSmemBytes = kOffStage + kStages * kTileBytes + 1024;  // + room to align the base
constexpr uint32_t kTmemCols = 256;           // S / P buffers at 0 and 64, O_tile at 128
constexpr uint32_t kColO = 128;
constexpr float kLog2eScale = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)

// Byte offset of 16-byte chunk c of row r in a K-major 128-byte-swizzled region.
__host__ __device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * kRowBytes + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// 2^x (PTX ex2.approx, flushes subnormal results to zero; 2^-inf = 0).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
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

// S = Q K^T: three products A_hi B_hi + A_hi B_lo + A_lo B_hi over K = 64 (4 steps of 16).
__device__ __forceinline__ void mma_qk(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
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

// O_tile = P V: A = P from tensor memory (hi in columns 0..31 of the buffer, lo in 32..63, two
// keys per column), B = V^T hi / lo from shared memory; three products over K = 64 keys.
__device__ __forceinline__ void mma_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_hi, uint32_t v_lo,
                                       uint32_t idesc) {
  const uint32_t as[3] = {p_tmem, p_tmem, p_tmem + 32}, bs[3] = {v_hi, v_lo, v_hi};
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    const uint64_t bd = tc::sw128_desc(bs[p]);
#pragma unroll
    for (int k = 0; k < 4; ++k)  // 16 keys = 8 tensor-memory columns of A, 32 bytes of a B row
      tc::tc_mma_ts(d_tmem, as[p] + 8 * k, bd + (uint64_t)(2 * k), idesc, (p > 0 || k > 0) ? 1u : 0u);
  }
}

// Bounded wait for phase `parity` of an mbarrier; false (and the error word set) on timeout or
// after another thread of the CTA gave up.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, uint32_t* error, unsigned long long wait_ns,
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

// Wait (bounded, no error) for phase `parity`: used only to drain work already in flight.
__device__ __forceinline__ void drain_bar(uint32_t bar, uint32_t parity, unsigned long long wait_ns) {
  const unsigned long long t0 = gtimer();
  while (!mbar_try(bar, parity) && gtimer() - t0 < wait_ns) {
  }
}

}  // namespace attn

// kc / vc: the slot's K / V cache of this layer ([pos][kv_dim]); img: [kv_heads][tile_stride]
// tile images of attn::kTileBytes.  Grid (kv_heads, p_last / 64 + 1), 128 threads.
__global__ void __launch_bounds__(128) k_kv_tiles(const float* __restrict__ kc, const float* __restrict__ vc,
                                                  int kv_dim, int p_last, uint8_t* __restrict__ img,
                                                  int tile_stride) {
  using namespace attn;
  __shared__ float sv[kKeys][LE_HEAD_DIM + 1];
  grid_dep_launch();
  const int g = blockIdx.x, t = blockIdx.y, tid = threadIdx.x;
  const int key = tid >> 1, half = tid & 1;  // 2 threads per key row, 32 dims each
  const int p = t * kKeys + key;
  uint8_t* dst = img + ((size_t)g * tile_stride + t) * kTileBytes;
  grid_dep_wait();  // the chunk's own rows were appended by the previous kernel
  const size_t off = (size_t)p * kv_dim + (size_t)g * LE_HEAD_DIM + 32 * half;
  const bool live = p <= p_last;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 a = live ? *reinterpret_cast<const float4*>(kc + off + 8 * i) : z;
    const float4 b = live ? *reinterpret_cast<const float4*>(kc + off + 8 * i + 4) : z;
    uint4 hi, lo;
    split_bf16(a.x, a.y, hi.x, lo.x);
    split_bf16(a.z, a.w, hi.y, lo.y);
    split_bf16(b.x, b.y, hi.z, lo.z);
    split_bf16(b.z, b.w, hi.w, lo.w);
    const uint32_t o = swz(key, 4 * half + i);
    *reinterpret_cast<uint4*>(dst + o) = hi;
    *reinterpret_cast<uint4*>(dst + kPartBytes + o) = lo;
    const float4 va = live ? *reinterpret_cast<const float4*>(vc + off + 8 * i) : z;
    const float4 vb = live ? *reinterpret_cast<const float4*>(vc + off + 8 * i + 4) : z;
    float* r = &sv[key][32 * half + 8 * i];
    r[0] = va.x; r[1] = va.y; r[2] = va.z; r[3] = va.w;
    r[4] = vb.x; r[5] = vb.y; r[6] = vb.z; r[7] = vb.w;
  }
  __syncthreads();
  const int d = tid >> 1;  // V^T row: dimension d, keys 32 half .. 32 half + 31
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k0 = 32 * half + 8 * i;
    uint4 hi, lo;
    split_bf16(sv[k0 + 0][d], sv[k0 + 1][d], hi.x, lo.x);
    split_bf16(sv[k0 + 2][d], sv[k0 + 3][d], hi.y, lo.y);
    split_bf16(sv[k0 + 4][d], sv[k0 + 5][d], hi.z, lo.z);
    split_bf16(sv[k0 + 6][d], sv[k0 + 7][d], hi.w, lo.w);
    const uint32_t o = swz(d, 4 * half + i);
    *reinterpret_cast<uint4*>(dst + 2 * kPartBytes + o) = hi;
    *reinterpret_cast<uint4*>(dst + 3 * kPartBytes + o) = lo;
  }
}

// q: rotated queries [T][q_dim] (rows of the chunk, positions p0 ..); img: the layer's tile
// images (k_kv_tiles, keys 0 .. p0 + T - 1); out: [T][q_dim].
// Grid (kv_heads, ceil(T / 32)), 128 threads, attn::kSmemBytes of dynamic shared memory.
// expire (test only): thread 0 first waits on a barrier phase that nothing completes.
__global__ void __launch_bounds__(128) k_attn_prefill_tc5(const float* __restrict__ q, int q_dim,
                                                          const uint8_t* __restrict__ img, int tile_stride, int p0,
                                                          int T, float* __restrict__ out, uint32_t* error,
                                                          unsigned long long wait_ns, int expire) {
  using namespace attn;
  extern __shared__ uint8_t attn_smem_raw[];
  __shared__ __align__(8) unsigned long long s_bar[4];  // full[0], full[1], S ready, O_tile ready
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
  const int first_pos = p0 + tok0;  // tiles ending at or before it need no mask
  const uint32_t base = (smem_u32(attn_smem_raw) + 1023u) & ~1023u;
  const uint32_t bar_full0 = smem_u32(&s_bar[0]);
  const uint32_t bar_s = smem_u32(&s_bar[2]);
  const uint32_t bar_o = smem_u32(&s_bar[3]);
  const uint32_t row = (uint32_t)tid;  // MMA row / tensor-memory lane of this thread
  const uint8_t* tiles = img + (size_t)g * tile_stride * kTileBytes;
  auto stage = [&](int j) { return base + kOffStage + (uint32_t)((j & 1) * kTileBytes); };

  grid_dep_launch();
  if (tid == 0) {
    s_abort = 0u;
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&s_bar[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&s_tmem), kTmemCols);
    tc::tmem_relinquish();
  }
  grid_dep_wait();  // q and the tile images come from the previous kernels of the step
  int copies = 0;   // thread 0: tile copies issued (tile j into stage j & 1)
  if (tid == 0) {
    for (; copies < min(kStages, ntiles); ++copies) {
      mbar_expect_tx(bar_full0 + 8 * copies, kTileBytes);
      bulk_g2s(stage(copies), tiles + (size_t)copies * kTileBytes, kTileBytes, bar_full0 + 8 * copies);
    }
  }

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
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // Q visible to the tensor core
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t t_lane = tmem + ((uint32_t)(32 * warp) << 16);  // this warp's lanes, column 0
  const uint32_t idesc = tc::idesc_bf16(64);

  // thread 0: S_j = Q K_j^T into S buffer j & 1, once tile j has landed
  int n_mma = 0;  // thread 0: MMA groups committed (to bar_s or bar_o)
  uint32_t last_bar = 0, last_parity = 0;
  auto issue_s = [&](int j) {
    if (s_abort) return;
    if (!attn::wait_bar(bar_full0 + 8 * (j & 1), (uint32_t)(j >> 1) & 1u, error, wait_ns, &s_abort)) return;
    tc::tc_fence_after();
    const uint32_t st = stage(j);
    attn::mma_qk(tmem + 64u * (uint32_t)(j & 1), base + kOffQ, base + kOffQ + kQBytes, st, st + kPartBytes, idesc);
    tc::tc_commit(bar_s);
    ++n_mma;
    last_bar = bar_s;
    last_parity = (uint32_t)j & 1u;
  };
  // test only: phase 0 of the O_tile barrier completes only after the first P V product, which
  // is issued after this wait, so the wait runs out (the tile copies are in flight meanwhile)
  if (expire && tid == 0) attn::wait_bar(bar_o, 0u, error, wait_ns, &s_abort);
  if (tid == 0) issue_s(0);

  float o[LE_HEAD_DIM];
#pragma unroll
  for (int d = 0; d < LE_HEAD_DIM; ++d) o[d] = 0.0f;
  float m = -INFINITY, l = 0.0f;  // running max (log2 units) and sum of this row

  for (int j = 0; j < ntiles; ++j) {
    const int k0 = j * kKeys;
    const uint32_t t_s = t_lane + 64u * (uint32_t)(j & 1);
    attn::wait_bar(bar_s, (uint32_t)j & 1u, error, wait_ns, &s_abort);
    tc::tc_fence_after();
    // ---- online softmax of this thread's row; P (bf16 hi / lo) replaces S ----
    float s[kKeys];
    {
      uint32_t r0[32], r1[32];
      tc::tmem_ld32(t_s, r0);
      tc::tmem_ld32(t_s + 32, r1);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        s[i] = __uint_as_float(r0[i]) * kLog2eScale;
        s[32 + i] = __uint_as_float(r1[i]) * kLog2eScale;
      }
    }
    if (k0 + kKeys - 1 > first_pos) {  // the causal edge (and the zero keys past p_last) is here
#pragma unroll
      for (int i = 0; i < kKeys; ++i) s[i] = k0 + i <= qpos ? s[i] : -INFINITY;
    }
    float mt = s[0];
#pragma unroll
    for (int i = 1; i < kKeys; ++i) mt = fmaxf(mt, s[i]);
    const float mn = fmaxf(m, mt);  // tile 0 holds key 0 <= every query: finite from there on
    const float alpha = attn::exp2_approx(m - mn);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kKeys; ++i) {
      s[i] = attn::exp2_approx(s[i] - mn);
      sum += s[i];
    }
    l = l * alpha + sum;
    m = mn;
#pragma unroll
    for (int c = 0; c < 2; ++c) {  // keys 32 c .. 32 c + 31: columns 16 c .. of hi, 32 + 16 c .. of lo
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) split_bf16(s[32 * c + 2 * e], s[32 * c + 2 * e + 1], hi[e], lo[e]);
      attn::tmem_st16(t_s + 16u * c, hi);
      attn::tmem_st16(t_s + 32u + 16u * c, lo);
    }
    tc::tmem_wait_st();
    tc::tc_fence_before();
    __syncthreads();
    // ---- O_tile = P V_j, then S_{j+1} ----
    if (tid == 0 && !s_abort) {
      tc::tc_fence_after();
      const uint32_t st = stage(j);
      attn::mma_pv(tmem + kColO, tmem + 64u * (uint32_t)(j & 1), st + 2 * kPartBytes, st + 3 * kPartBytes, idesc);
      tc::tc_commit(bar_o);
      ++n_mma;
      last_bar = bar_o;
      last_parity = (uint32_t)j & 1u;
      if (j + 1 < ntiles) issue_s(j + 1);
    }
    attn::wait_bar(bar_o, (uint32_t)j & 1u, error, wait_ns, &s_abort);
    tc::tc_fence_after();
    {
      uint32_t r0[32], r1[32];
      tc::tmem_ld32(t_lane + kColO, r0);
      tc::tmem_ld32(t_lane + kColO + 32, r1);
      tc::tmem_wait_ld();
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        o[d] = fmaf(o[d], alpha, __uint_as_float(r0[d]));
        o[32 + d] = fmaf(o[32 + d], alpha, __uint_as_float(r1[d]));
      }
    }
    // stage j & 1 is free (S_j and O_tile_j have completed): tile j + 2 goes there
    if (tid == 0 && copies < ntiles && !s_abort) {
      mbar_expect_tx(bar_full0 + 8 * (copies & 1), kTileBytes);
      bulk_g2s(stage(copies), tiles + (size_t)copies * kTileBytes, kTileBytes, bar_full0 + 8 * (copies & 1));
      ++copies;
    }
    tc::tc_fence_before();
    __syncthreads();  // O_tile read before the next P V overwrites it
  }
  if (tok0 + lane < T) {
    const float inv = 1.0f / l;
    float* orow = out + (size_t)(tok0 + lane) * q_dim + (size_t)h * LE_HEAD_DIM;
#pragma unroll
    for (int d = 0; d < LE_HEAD_DIM; d += 4)
      *reinterpret_cast<float4*>(orow + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
  }
  // Normally every MMA and copy has been waited for.  After a timeout, thread 0 waits (bounded)
  // for its last MMA commit (which covers all its earlier MMAs) and for the copies it issued
  // beyond the tiles whose copies were waited for, before the shared and tensor memory go.
  if (s_abort && tid == 0) {
    if (n_mma > 0) attn::drain_bar(last_bar, last_parity, wait_ns);
    for (int c = max(0, copies - kStages); c < copies; ++c) attn::drain_bar(bar_full0 + 8 * (c & 1), (uint32_t)(c >> 1) & 1u, wait_ns);
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
