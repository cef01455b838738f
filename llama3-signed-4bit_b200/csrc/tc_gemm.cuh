// Tensor-core (tcgen05) GEMM over block-128 4-bit weights, for several tokens at once: batched
// decode and prefill (src/llama_engine.cpp:935-1042 run for T tokens; the GEMV is
// signed_4bit_b128_gemv, :233-357).
//
//   y[t][n] = sum_b ( min[n][b] * xs[t][b]  +  step[n][b] * sum_{k in b} q[n][k] * x[t][k] )
//
// One CTA (10 warps, one per SM, persistent over work units) computes a tile of 128 weight rows
// for up to 64 tokens over a range of 128-wide K blocks:
//
//   * warp 0 (one lane) streams, per K block, the activation image of the token tile (the 64
//     token rows as bf16 hi and lo parts, x = hi + lo, hi = bf16(x), lo = bf16(x - hi), already
//     in the UMMA K-major 128-byte-swizzled layout, plus the tokens' block sums) and the tile's
//     weight record (nibbles + scales) with two 1-D bulk copies into a 4-stage shared-memory ring;
//   * warps 2..9 (the row warps, thread = weight row) turn each record's nibbles into bf16 codes
//     q (exact: 0..15) and write them into tensor memory (tcgen05.st) as the MMA's A operand;
//   * warp 1 (one lane) issues, per 16-wide K step, two tcgen05.mma kind::f16 with A = q from
//     tensor memory: D_hi += q . x_hi and D_lo += q . x_lo (fp32 accumulators in tensor memory,
//     one pair per K block, double buffered);
//   * the row warps then read D_hi and D_lo back (tcgen05.ld) and apply the block's scales in
//     fp32: acc[t] += min * xs[t] + step * (D_hi[t] + D_lo[t]) (the reference's factored form).
//
// Products q * x_hi and q * x_lo are exact in fp32; the only rounding beyond fp32 accumulation
// is lo's own bf16 rounding (relative 2^-17 of x).  Work units end with a mode-specific epilogue:
// plain rows (split-K partials or logits), RoPE + KV-cache append for the q|k|v rows, or
// SiLU(gate) * up for interleaved gate/up tiles.
//
// Weight records are built at load time from the LLM4S128 matrices: per (row tile, K block)
// 8704 bytes: [0, 8192) row r's 64 nibble bytes at r*64, its 16-byte chunk c stored at chunk
// position c ^ ((r >> 1) & 3) (conflict-free 16-byte shared loads); [8192, 8704) row r's
// (step | min << 16) at 8192 + 4r.  Rows past the matrix are zero.
//
// Activation images are written by k_tc_stage: per (token tile, K block) 33024 bytes: four
// 8192-byte atoms (hi k 0..63, hi k 64..127, lo k 0..63, lo k 64..127), each 64 token rows of
// 128 bytes with 16-byte chunk c of row t at chunk position c ^ (t & 7) (the 128-byte swizzle
// of the UMMA canonical K-major layout, 8-row groups 1024 bytes apart), then the 64 tokens'
// block sums (fp32).
//
// All mbarrier waits are bounded in time: on timeout the kernel records an error word and every
// role drains, so the host sees an error instead of a hang.
#pragma once

#include <cuda_bf16.h>

#include "persistent.cuh"

namespace le {
namespace tc {

constexpr int kM = 128;                  // weight rows per tile (UMMA M)
constexpr int kTok = 64;                 // tokens per tile
constexpr int kNibBytes = kM * 64;       // nibbles of one (tile, K block)
constexpr int kRecBytes = kNibBytes + kM * 4;
constexpr int kAtom = kTok * 128;        // one 64-wide K slice of 64 token rows (bf16, swizzled)
constexpr int kStages = 4;
constexpr int kImgBytes = 4 * kAtom + kTok * 4;  // activation image of one (token tile, K block)
constexpr int kOffXs = 4 * kAtom;        // stage: hi0 | hi1 | lo0 | lo1 | xs | record
constexpr int kOffRec = kImgBytes;
constexpr int kStageTx = kImgBytes + kRecBytes;
constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
constexpr int kXchStride = kM + 1;       // exchange rows of 128 floats, padded
constexpr int kXchBytes = 2 * 32 * kXchStride * 4;
constexpr int kWarps = 10;
constexpr int kThreads = 32 * kWarps;
constexpr int kTmemCols = 512;           // A[2] (64 cols each) | D[2] (hi 64 | lo 64 each)
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kXchBytes + 256;

enum Mode : int { MODE_ROWS = 0, MODE_QKV = 1, MODE_SWIGLU = 2 };

struct Args {
  const uint8_t* recs;   // [tiles][kb_total][kRecBytes]
  const uint8_t* img;    // [tok_tiles][kb_total][kImgBytes]
  int tiles, kb_total, tok_tiles, splits, kb_split;
  int T, nt;             // valid tokens, MMA N (16..64)
  int N;                 // valid output rows (MODE_ROWS / MODE_QKV), ffn (MODE_SWIGLU)
  int mode;
  float* out;            // ROWS: out[(split * T + t) * ldo + n]; QKV: q rows; SWIGLU: act
  int ldo;
  size_t split_stride;   // ROWS: floats between split planes
  // MODE_QKV
  const int32_t* pos;
  const int32_t* slot;
  const float* rope_cos;
  const float* rope_sin;
  float* kc;             // cache of slot 0 at this layer; slot s at + s * slot_stride
  float* vc;
  size_t slot_stride;
  int q_rows, kv_dim;
  uint32_t* error;       // set to a nonzero code on a wait timeout
};

// ---------------------------------------------------------------------------------------------
// PTX wrappers (tcgen05, TMA)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate), M = 128.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 bytes, 8-row groups
// 1024 bytes apart (stride byte offset), descriptor version 1 (tcgen05).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
}

// bf16x2 of the two nibbles of byte i of w (element 2i in the low half, 2i+1 in the high half).
// prmt puts byte i of w and byte i of (w >> 4) into the two halves, the mask keeps one nibble in
// each and sets the bf16 exponent of 128, so the halves read 128 + q; the fma removes the 128.
template <int I>
__device__ __forceinline__ uint32_t nib_pair_bf16(uint32_t w, uint32_t w4) {
  uint32_t t;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(t) : "r"(w), "r"(w4), "n"(I | (I << 4) | ((I + 4) << 8) | ((I + 4) << 12)));
  t = (t & 0x000F000Fu) | 0x43004300u;
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(t), "r"(0x3F803F80u), "r"(0xC300C300u));
  return r;
}

struct Shared {
  uint32_t base;   // 1024-aligned shared address of stage 0
  uint32_t xch;    // exchange buffer
  uint32_t bar;    // barriers: full[4] empty[4] afull[2] dfull[2] dempty[2] final xch[2]
};
__device__ __forceinline__ uint32_t bar_full(const Shared& S, int s) { return S.bar + 8 * s; }
__device__ __forceinline__ uint32_t bar_empty(const Shared& S, int s) { return S.bar + 8 * (kStages + s); }
__device__ __forceinline__ uint32_t bar_afull(const Shared& S, int a) { return S.bar + 8 * (2 * kStages + a); }
__device__ __forceinline__ uint32_t bar_dfull(const Shared& S, int a) { return S.bar + 8 * (2 * kStages + 2 + a); }
__device__ __forceinline__ uint32_t bar_dempty(const Shared& S, int a) { return S.bar + 8 * (2 * kStages + 4 + a); }
__device__ __forceinline__ uint32_t bar_final(const Shared& S) { return S.bar + 8 * (2 * kStages + 6); }
__device__ __forceinline__ uint32_t bar_xch(const Shared& S, int h) { return S.bar + 8 * (2 * kStages + 7 + h); }

// Bounded wait on an mbarrier phase.  Returns false when the launch has failed (here or in
// another role); the first timeout records `where`.
__device__ __forceinline__ bool wait_bar(const Args& A, volatile uint32_t* abort_flag, uint32_t bar, uint32_t parity,
                                         uint32_t where) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > kWaitNs) {
      *abort_flag = 1u;
      atomicCAS(A.error, 0u, where);
      return false;
    }
  }
}

struct Unit {
  int tile, tt, split, kb0, kb1;
};
__device__ __forceinline__ Unit unit_of(const Args& A, int u) {
  Unit U;
  const int per_tile = A.tok_tiles * A.splits;
  U.tile = u / per_tile;
  const int r = u - U.tile * per_tile;
  U.tt = r / A.splits;
  U.split = r - U.tt * A.splits;
  U.kb0 = U.split * A.kb_split;
  U.kb1 = min(A.kb_total, U.kb0 + A.kb_split);
  return U;
}

// Unit epilogue of the row warps.  Thread (q, h, lane) owns weight row r = 32q + lane of the
// tile and tokens 32h .. 32h+31 of the token tile.
// The exchange between the four row warps of a token half uses an mbarrier (bounded wait), so a
// warp that has given up after a timeout cannot leave the others blocked.
__device__ __forceinline__ bool xch_sync(const Args& A, volatile uint32_t* abort_flag, const Shared& S, int h,
                                         int& xph) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_n(bar_xch(S, h), 1);
  const bool ok = __all_sync(0xffffffffu, wait_bar(A, abort_flag, bar_xch(S, h), (uint32_t)(xph & 1), 9));
  ++xph;
  return ok;
}

__device__ __forceinline__ bool emit_unit(const Args& A, volatile uint32_t* abort_flag, const Shared& S,
                                          const Unit& U, int r, int h, int& xph, const float (&acc)[32]) {
  const int tok0 = U.tt * kTok + 32 * h;
  if (A.mode == MODE_ROWS) {
    const int n = U.tile * kM + r;
    if (n >= A.N) return true;
    float* o = A.out + (size_t)U.split * A.split_stride + n;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int t = tok0 + i;
      if (t < A.T) o[(size_t)t * A.ldo] = acc[i];
    }
    return true;
  }
  // exchange through shared memory: xch[h][i][r]
  const uint32_t xb = S.xch + (uint32_t)(h * 32 * kXchStride) * 4u;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(xb + (uint32_t)(i * kXchStride + r) * 4u), "f"(acc[i]) : "memory");
  if (!xch_sync(A, abort_flag, S, h, xph)) return false;
  if (A.mode == MODE_QKV) {
    const int n = U.tile * kM + r;
    const int i2 = r & 31;
    const bool second = (r & 32) != 0;
    const int partner = r ^ 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int t = tok0 + i;
      if (t >= A.T || n >= A.N) continue;
      const float own = acc[i];
      const float oth = ldsf(xb + (uint32_t)(i * kXchStride + partner) * 4u);
      if (n < A.q_rows + A.kv_dim) {
        const int p = A.pos[t];
        const float c = A.rope_cos[p * 32 + i2], s = A.rope_sin[p * 32 + i2];
        // apply_rope (src/llama_engine.cpp:120-151): (x0, x1) -> (x0 c - x1 s, x0 s + x1 c)
        const float x0 = second ? oth : own, x1 = second ? own : oth;
        const float v = second ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                               : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        if (n < A.q_rows) {
          A.out[(size_t)t * A.ldo + n] = v;
        } else {
          A.kc[(size_t)A.slot[t] * A.slot_stride + (size_t)p * A.kv_dim + (n - A.q_rows)] = v;
        }
      } else {
        const int p = A.pos[t];
        A.vc[(size_t)A.slot[t] * A.slot_stride + (size_t)p * A.kv_dim + (n - A.q_rows - A.kv_dim)] = own;
      }
    }
  } else {  // MODE_SWIGLU: rows 0..63 gate, 64..127 up of the same 64 ffn rows
    if (r < 64) {
      const int j = U.tile * 64 + r;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int t = tok0 + i;
        if (t >= A.T || j >= A.N) continue;
        const float g = acc[i];
        const float u = ldsf(xb + (uint32_t)(i * kXchStride + r + 64) * 4u);
        A.out[(size_t)t * A.ldo + j] = (g / (1.0f + expf(-g))) * u;
      }
    }
  }
  return xch_sync(A, abort_flag, S, h, xph);  // the exchange rows are reused by the next unit
}

__global__ void __launch_bounds__(kThreads, 1) k_tc_gemm(Args A) {
  extern __shared__ __align__(1024) uint8_t tc_smem[];
  __shared__ uint32_t s_tmem;
  __shared__ volatile uint32_t s_abort;
  Shared S;
  S.base = (smem_u32(tc_smem) + 1023u) & ~1023u;
  S.xch = S.base + kStages * kStageBytes;
  S.bar = S.xch + kXchBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = A.tiles * A.tok_tiles * A.splits;

  if (threadIdx.x == 0) {
    s_abort = 0u;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full(S, s), 1);
      mbar_init(bar_empty(S, s), 1 + 8);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_afull(S, a), 8);
      mbar_init(bar_dfull(S, a), 1);
      mbar_init(bar_dempty(S, a), 8);
    }
    mbar_init(bar_final(S), 1);
    mbar_init(bar_xch(S, 0), 4);
    mbar_init(bar_xch(S, 1), 4);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&s_tmem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int g = 0;
      for (int u = blockIdx.x; u < n_units && !s_abort; u += gridDim.x) {
        const Unit U = unit_of(A, u);
        for (int kb = U.kb0; kb < U.kb1; ++kb, ++g) {
          const int s = g % kStages, n = g / kStages;
          if (g >= kStages && !wait_bar(A, &s_abort, bar_empty(S, s), (n - 1) & 1, 1)) break;
          const uint32_t st = S.base + s * kStageBytes;
          const uint32_t fb = bar_full(S, s);
          mbar_expect_tx(fb, kStageTx);
          bulk_g2s(st, A.img + ((size_t)U.tt * A.kb_total + kb) * kImgBytes, kImgBytes, fb);
          bulk_g2s(st + kOffRec, A.recs + ((size_t)U.tile * A.kb_total + kb) * kRecBytes, kRecBytes, fb);
        }
      }
      // drain: every issued stage must have landed before the CTA may exit
      const int issued = g;
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int last = issued - 1 - ((issued - 1 - s) % kStages);  // last fill of stage s
        wait_bar(A, &s_abort, bar_full(S, s), (last / kStages) & 1, 2);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_bf16(A.nt);
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Unit U = unit_of(A, u);
        for (int kb = U.kb0; kb < U.kb1; ++kb, ++g) {
          const int s = g % kStages, n = g / kStages, a = g & 1, na = g >> 1;
          ok = wait_bar(A, &s_abort, bar_full(S, s), n & 1, 3) && wait_bar(A, &s_abort, bar_afull(S, a), na & 1, 4) &&
               (g < 2 || wait_bar(A, &s_abort, bar_dempty(S, a), (na - 1) & 1, 5));
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = S.base + s * kStageBytes;
          const uint32_t d_hi = tmem + 128 + a * 128, d_lo = d_hi + 64;
          const uint32_t a_t = tmem + a * 64;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t b_hi = st + (k >> 2) * kAtom + (k & 3) * 32;
            tc_mma_ts(d_hi, a_t + 8 * k, sw128_desc(b_hi), idesc, k > 0);
            tc_mma_ts(d_lo, a_t + 8 * k, sw128_desc(b_hi + 2 * kAtom), idesc, k > 0);
          }
          tc_commit(bar_empty(S, s));
          tc_commit(bar_dfull(S, a));
        }
      }
      // all issued MMAs complete before the tensor memory is released
      tc_commit(bar_final(S));
      wait_bar(A, &s_abort, bar_final(S), 0, 6);
    }
  } else {
    // ---------------- row warps: dequantise into tensor memory, per-block epilogue ----------------
    const int q = warp & 3;
    const int h = warp < 6 ? 0 : 1;
    const int r = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const int sw = (r >> 1) & 3;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
    int g = 0, xph = 0;
    bool ok = true;
    Unit prev{};
    bool prev_last = false;
    // per-block epilogue of block gp (stage sp, buffer ap)
    auto epilogue = [&](int gp) -> bool {
      const int sp = gp % kStages, ap = gp & 1, nap = gp >> 1;
      // lanes leave the poll at different times; the vote reconverges the warp (tcgen05.ld is
      // warp-aligned) and makes a timeout warp-uniform
      if (!__all_sync(0xffffffffu, wait_bar(A, &s_abort, bar_dfull(S, ap), nap & 1, 7))) return false;
      tc_fence_after();
      uint32_t vh[32], vl[32];
      const uint32_t dcol = tmem + lane_base + 128 + ap * 128 + 32 * h;
      tmem_ld32(dcol, vh);
      tmem_ld32(dcol + 64, vl);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_n(bar_dempty(S, ap), 1);
      const uint32_t st = S.base + sp * kStageBytes;
      const uint32_t sc = lds32(st + kOffRec + kNibBytes + 4 * r);
      const float step = bf16_bits_to_f32(sc & 0xFFFFu), mn = bf16_bits_to_f32(sc >> 16);
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const uint4 x4 = lds128(st + kOffXs + 4 * (32 * h + i));
        const float xs[4] = {__uint_as_float(x4.x), __uint_as_float(x4.y), __uint_as_float(x4.z),
                             __uint_as_float(x4.w)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float d = __uint_as_float(vh[i + j]) + __uint_as_float(vl[i + j]);
          acc[i + j] = fmaf(step, d, fmaf(mn, xs[j], acc[i + j]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_n(bar_empty(S, sp), 1);
      return true;
    };
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Unit U = unit_of(A, u);
      for (int kb = U.kb0; kb < U.kb1; ++kb, ++g) {
        const int s = g % kStages, n = g / kStages, a = g & 1;
        if (!__all_sync(0xffffffffu, wait_bar(A, &s_abort, bar_full(S, s), n & 1, 8))) { ok = false; break; }
        // dequantise this thread's half of the block row into A[a]
        const uint32_t rec = S.base + s * kStageBytes + kOffRec + 64 * r;
        const uint4 c0 = lds128(rec + (uint32_t)(((2 * h) ^ sw) << 4));
        const uint4 c1 = lds128(rec + (uint32_t)(((2 * h + 1) ^ sw) << 4));
        const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        uint32_t v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t w4 = w[j] >> 4;
          v[4 * j + 0] = nib_pair_bf16<0>(w[j], w4);
          v[4 * j + 1] = nib_pair_bf16<1>(w[j], w4);
          v[4 * j + 2] = nib_pair_bf16<2>(w[j], w4);
          v[4 * j + 3] = nib_pair_bf16<3>(w[j], w4);
        }
        tmem_st32(tmem + lane_base + a * 64 + 32 * h, v);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_n(bar_afull(S, a), 1);
        if (g > 0) {
          if (!epilogue(g - 1)) { ok = false; break; }
          if (prev_last) {
            if (!emit_unit(A, &s_abort, S, prev, r, h, xph, acc)) { ok = false; break; }
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
          }
        }
        prev = U;
        prev_last = (kb + 1 == U.kb1);
      }
    }
    if (ok && g > 0 && epilogue(g - 1) && prev_last) emit_unit(A, &s_abort, S, prev, r, h, xph, acc);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Weight record builder: rows [0, N) of W go to tile rows dest(n) = row0 + (n / G) * 128 + off +
// n % G of a record arena with kb_total = W.K / 128 blocks per tile (G = 128, off = 0 for plain
// and concatenated matrices; G = 64, off = 0 / 64 for the gate / up halves of gate-up tiles).
// ---------------------------------------------------------------------------------------------
__global__ void k_tc_repack(QMat W, uint8_t* __restrict__ recs, int row0, int G, int off) {
  const int kbt = W.K >> 7;
  const size_t total = (size_t)W.N * kbt * 4;  // one thread per 16-byte nibble chunk
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i & 3);
    const size_t nb = i >> 2;
    const int n = (int)(nb / kbt), kb = (int)(nb % kbt);
    const int dr = row0 + (n / G) * kM + off + n % G;
    const int tile = dr / kM, rr = dr % kM;
    uint8_t* rec = recs + ((size_t)tile * kbt + kb) * kRecBytes;
    const uint4 src = *reinterpret_cast<const uint4*>(W.nib + (size_t)n * (W.K >> 1) + kb * 64 + c * 16);
    *reinterpret_cast<uint4*>(rec + rr * 64 + ((c ^ ((rr >> 1) & 3)) << 4)) = src;
    if (c == 0) {
      const size_t blk = (size_t)n * kbt + kb;
      *reinterpret_cast<uint32_t*>(rec + kNibBytes + rr * 4) = (uint32_t)W.step[blk] | ((uint32_t)W.mn[blk] << 16);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Activation staging: for token row t (one CTA of 256 threads), optionally fold split-K partial
// sums into the residual x (x += sum_s part[s]) and write x back, optionally rms-normalise with
// gamma (rms_norm, src/llama_engine.cpp:87-115), then write row t of the activation image (bf16
// hi / lo parts in the swizzled atom layout, and the 128-wide block sums of compute_x_block_sums,
// :496-521).  K is a multiple of 2048; a thread handles runs of 8 consecutive elements.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_tc_stage(float* __restrict__ x, int ldx, const float* __restrict__ part,
                                                  int nsplit, size_t split_stride, const float* __restrict__ gamma,
                                                  int K, uint8_t* __restrict__ img) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int runs = K / 2048;  // runs of 8 per thread: 1..4
  const int kbt = K >> 7;
  float v[32];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j >= runs) break;
    const int i0 = j * 2048 + threadIdx.x * 8;
    float* xp = x + (size_t)t * ldx + i0;
    const float4 a = *reinterpret_cast<const float4*>(xp), b = *reinterpret_cast<const float4*>(xp + 4);
    float e[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (nsplit > 0) {
      const float* pp = part + (size_t)t * K + i0;
      float s8[8];
      {
        const float4 p0 = *reinterpret_cast<const float4*>(pp), p1 = *reinterpret_cast<const float4*>(pp + 4);
        s8[0] = p0.x; s8[1] = p0.y; s8[2] = p0.z; s8[3] = p0.w; s8[4] = p1.x; s8[5] = p1.y; s8[6] = p1.z; s8[7] = p1.w;
      }
      for (int sp = 1; sp < nsplit; ++sp) {
        const float4 p0 = *reinterpret_cast<const float4*>(pp + sp * split_stride);
        const float4 p1 = *reinterpret_cast<const float4*>(pp + sp * split_stride + 4);
        s8[0] += p0.x; s8[1] += p0.y; s8[2] += p0.z; s8[3] += p0.w;
        s8[4] += p1.x; s8[5] += p1.y; s8[6] += p1.z; s8[7] += p1.w;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] += s8[k];
      *reinterpret_cast<float4*>(xp) = make_float4(e[0], e[1], e[2], e[3]);
      *reinterpret_cast<float4*>(xp + 4) = make_float4(e[4], e[5], e[6], e[7]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[j * 8 + k] = e[k];
      ss = fmaf(e[k], e[k], ss);
    }
  }
  if (gamma) {
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)K + 1e-5f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= runs) break;
      const int i0 = j * 2048 + threadIdx.x * 8;
#pragma unroll
      for (int k = 0; k < 8; ++k) v[j * 8 + k] = __fmul_rn(__fmul_rn(v[j * 8 + k], gamma[i0 + k]), inv);
    }
  }
  const int tt = t / kTok, tr = t % kTok;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j >= runs) break;
    const int i0 = j * 2048 + threadIdx.x * 8;
    uint32_t hw[4], lw[4];
    float bs = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      const float a0 = v[j * 8 + k], a1 = v[j * 8 + k + 1];
      const __nv_bfloat162 hh = __floats2bfloat162_rn(a0, a1);
      const __nv_bfloat162 ll = __floats2bfloat162_rn(a0 - __low2float(hh), a1 - __high2float(hh));
      hw[k / 2] = *reinterpret_cast<const uint32_t*>(&hh);
      lw[k / 2] = *reinterpret_cast<const uint32_t*>(&ll);
      bs += a0 + a1;
    }
    const int kb = i0 >> 7, kk = i0 & 127;
    uint8_t* im = img + ((size_t)tt * kbt + kb) * kImgBytes;
    const int atom = kk >> 6, c = (kk & 63) >> 3;
    const size_t o = (size_t)atom * kAtom + tr * 128 + ((c ^ (tr & 7)) << 4);
    *reinterpret_cast<uint4*>(im + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(im + 2 * kAtom + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    // 16 threads cover one 128-block
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o2);
    if ((threadIdx.x & 15) == 0) reinterpret_cast<float*>(im + kOffXs)[tr] = bs;
  }
}

}  // namespace tc
}  // namespace le
