// Tensor-core (tcgen05) GEMM over block-128 4-bit weights, for several tokens at once: batched
// decode and prefill (src/llama_engine.cpp:935-1042 run for T tokens; the GEMV is
// signed_4bit_b128_gemv, :233-357).
//
//   y[t][n] = sum_b ( min[n][b] * xs[t][b]  +  step[n][b] * sum_{k in b} q[n][k] * x[t][k] )
//
// One CTA (one per SM, persistent over work units) computes a tile of 128 weight rows for a unit
// of 64 tokens (or 128: two-tile units, Geo<2>) over a range of 128-wide K blocks, as a pipeline
// over K blocks (described here for 64-token units; Geo<P> gives the two-tile differences):
//
//   * warp 0 (one lane) streams, per K block, the activation image of the token tile (the 64
//     token rows as bf16 hi and lo parts, x = hi + lo, hi = bf16(x), lo = bf16(x - hi), already
//     in the UMMA K-major 128-byte-swizzled layout, plus the tokens' block sums) and the tile's
//     weight record (nibbles + scales) with two 1-D bulk copies into a 5-stage shared-memory
//     ring, and prefetches the records of later blocks into L2;
//   * warps 3..10 (dequantisers, two sets taking alternate blocks, thread = weight row; one set,
//     warps 3..6, for two-tile units) turn
//     each record's nibbles into bf16 codes q (exact: 0..15), write them into tensor memory
//     (tcgen05.st) as the MMA's A operand, and pass the block's scales and block sums to the
//     epilogue through a small side ring;
//   * warp 1 (one lane) issues, per 16-wide K step, one tcgen05.mma kind::f16 (M = 128, N = 128)
//     with A = q from tensor memory and B = the 64 tokens' hi rows stacked on their lo rows, into
//     an fp32 accumulator D in tensor memory (one per K block): D[t] = sum_k q . x_hi[t],
//     D[64 + t] = sum_k q . x_lo[t]; the MMAs' completion frees the stage, the A buffer and
//     signals the accumulator;
//   * warps 11..18 (epilogue, thread = weight row, 32 tokens each; warps 7..14 with 64 tokens
//     each in two-tile units) read D back (tcgen05.ld) and
//     apply the block's scales in fp32: acc[t] += min * xs[t] + step * (D[t] + D[64 + t]) (the
//     reference's factored form); at the end of a unit they store the rows (split-K partials,
//     projections or logits).
// A codes have four tensor-memory buffers, accumulators two.
//
// Products q * x_hi and q * x_lo are exact in fp32; the only rounding beyond fp32 accumulation
// is lo's own bf16 rounding (relative 2^-17 of x).
//
// Weight records are built at load time from the LLM4S128 matrices: per (row tile, K block)
// 8704 bytes: [0, 8192) row r's 64 nibble bytes at r*64, its 16-byte chunk c stored at chunk
// position c ^ ((r >> 1) & 3) (conflict-free 16-byte shared loads); [8192, 8704) row r's
// (step | min << 16) at 8192 + 4r.  Rows past the matrix are zero.
//
// Activation images are written by k_tc_stage: per (token tile, K block) 33024 bytes: four
// 8192-byte atoms (hi k 0..63, lo k 0..63, hi k 64..127, lo k 64..127), each 64 token rows of
// 128 bytes with 16-byte chunk c of row t at chunk position c ^ (t & 7) (the 128-byte swizzle
// of the UMMA canonical K-major layout, 8-row groups 1024 bytes apart; a hi atom and the lo atom
// after it form one 128-row B operand), then the 64 tokens' block sums (fp32).
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
constexpr int kImgBytes = 4 * kAtom + kTok * 4;  // activation image of one (token tile, K block)
constexpr int kOffXs = 4 * kAtom;        // image: hi0 | lo0 | hi1 | lo1 | xs
constexpr int kBufsA = 4;                // tensor-memory buffers of A codes (64 columns each)
constexpr int kBufsD = 2;                // accumulator buffers (128 columns)
constexpr int kTmemCols = 512;
constexpr int kDCol = kBufsA * 64;
constexpr uint32_t kSleepNs = 20000;    // suspend hint of a pending wait (the bound is checked between)
constexpr int kPrefetch = 8;             // records prefetched into L2 this many blocks ahead

// Shared-memory geometry for work units of P 64-token tiles.
//   P = 1 (decode-sized steps): a stage is one tile's activation image as stored (hi0 | lo0 |
//   hi1 | lo1 | xs), then the weight record; 5 stages, 8 side slots.  The MMA's B operand for a
//   16-wide K step is the tile's hi rows stacked on its lo rows (N = 128): accumulator columns
//   t and 64 + t hold token t's x_hi and x_lo products.
//   P = 2 (prefill-sized steps): a stage holds two tiles' images regrouped so that each 64-wide
//   K slice of hi (or lo) parts is one 128-row B operand: hi atoms [K 0..63: tile 0 | tile 1]
//   [K 64..127: tile 0 | tile 1], the lo atoms likewise, the two tiles' block sums, then the
//   record; two MMAs per 16-wide K step (x_hi, then x_lo, N = 128 tokens) accumulate into one
//   column per token, so the issuer's per-block bookkeeping serves twice the tokens.  3 stages
//   and 3 side slots are what fit.
template <int P>
struct Geo {
  static constexpr int kUnitTok = P * kTok;                   // tokens per unit
  static constexpr int kOffLo = P == 1 ? kAtom : 4 * kAtom;   // first lo atom of a stage
  static constexpr int kOffXs = P == 1 ? 4 * kAtom : 8 * kAtom;
  static constexpr int kOffRec = kOffXs + kUnitTok * 4;
  static constexpr int kStageTx = kOffRec + kRecBytes;
  static constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
  static constexpr int kStages = P == 1 ? 5 : 3;
  static constexpr int kSide = P == 1 ? 8 : 3;  // side ring: per block the rows' scales and block sums
  // Warps: 0 producer, 1 MMA issuer, 2 idle, then kDqSets sets of 4 dequantisers, then 8 epilogue
  // warps.  One set converts a block in ~0.5 us: two sets taking alternate blocks keep up with the
  // 0.77 us block period of one-tile units; one set suffices for the 1.06 us period of two-tile
  // units, which then run 15 warps (128 registers a thread instead of 96: no spilled accumulators,
  // and fewer warps beside the MMA issuer on its sub-partition).
  static constexpr int kDqSets = P == 1 ? 2 : 1;
  static constexpr int kEpiWarp0 = 3 + 4 * kDqSets;
  static constexpr int kWarps = kEpiWarp0 + 8;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kSideBytes = kM * 4 + kUnitTok * 4;
  static constexpr int kNumBars = 2 * kStages + kBufsA + kBufsD + 2 * kSide + 1;
  // 1024 bytes of slack to align the dynamic base (the swizzled operands need 1024-byte atoms)
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kSide * kSideBytes + (kNumBars * 8 + 63) / 64 * 64;
};
static_assert(Geo<1>::kOffRec == kImgBytes, "a one-tile stage starts with the image as stored");
// dynamic plus the kernel's 1 KB of static shared memory, within the 232448 bytes a CTA may opt into
static_assert(Geo<1>::kSmemBytes + 1024 <= 232448 && Geo<2>::kSmemBytes + 1024 <= 232448,
              "stages must fit one CTA's shared memory");

struct Args {
  const uint8_t* recs;   // [tiles][kb_total][kRecBytes]
  const uint8_t* img;    // [img_tiles][kb_total][kImgBytes]
  int tiles, kb_total, tok_tiles, splits, kb_split;  // tok_tiles: token groups (P tiles each)
  int img_tiles;         // 64-token tiles held by img (a unit's second tile may lie past them)
  int T;                 // valid tokens
  int N;                 // valid output rows
  float* out;            // out[split * split_stride + t * ldo + n]
  int ldo;
  size_t split_stride;
  uint32_t* error;       // set to a nonzero code on a wait timeout
  unsigned long long* trace;  // optional: CTA 0's pipeline events, [kTraceEvents][kTraceBlocks]
  unsigned long long wait_ns;  // bound on every wait
  int expire;            // test only: nonzero makes the MMA issuer wait on a barrier nothing completes
  int swiglu;            // gate-up tiles (gate / up rows interleaved): store SiLU(gate) * up per ffn row
};

// Pipeline trace (diagnostics): globaltimer stamps of CTA 0 for its first kTraceBlocks blocks.
// 0: copies issued, 1: MMA inputs ready (waits passed), 2: dequantiser sees the stage,
// 3: A codes written, 4: epilogue sees the accumulator, 5: epilogue done with the block,
// 6: MMAs issued, 7: commit issued, 8: MMA loop top, 9: MMA issuer past the A-codes wait.
constexpr int kTraceEvents = 10;
constexpr int kTraceBlocks = 256;
__device__ __forceinline__ void trace_ev(const Args& A, int ev, int g) {
  if (A.trace && blockIdx.x == 0 && g < kTraceBlocks && (threadIdx.x & 31) == 0)
    A.trace[ev * kTraceBlocks + g] = gtimer();
}

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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
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

template <int P>
struct Shared {
  uint32_t base;   // 1024-aligned shared address of stage 0
  uint32_t side;   // side ring
  uint32_t bar;    // barriers
};
// barrier index layout: full[S] done[S] afull[BA] dempty[BD] sfull[side] sempty[side] final.
// done[g % S] completes when the MMAs of block g have: the stage, the A buffer of block g and
// its accumulator are then free or ready (one tcgen05.commit serves all three).
template <int P>
__device__ __forceinline__ uint32_t bar_full(const Shared<P>& S, int s) { return S.bar + 8 * s; }
template <int P>
__device__ __forceinline__ uint32_t bar_done(const Shared<P>& S, int s) {
  return S.bar + 8 * (Geo<P>::kStages + s);
}
template <int P>
__device__ __forceinline__ uint32_t bar_afull(const Shared<P>& S, int b) {
  return S.bar + 8 * (2 * Geo<P>::kStages + b);
}
template <int P>
__device__ __forceinline__ uint32_t bar_dempty(const Shared<P>& S, int b) {
  return S.bar + 8 * (2 * Geo<P>::kStages + kBufsA + b);
}
template <int P>
__device__ __forceinline__ uint32_t bar_sfull(const Shared<P>& S, int j) {
  return S.bar + 8 * (2 * Geo<P>::kStages + kBufsA + kBufsD + j);
}
template <int P>
__device__ __forceinline__ uint32_t bar_sempty(const Shared<P>& S, int j) {
  return S.bar + 8 * (2 * Geo<P>::kStages + kBufsA + kBufsD + Geo<P>::kSide + j);
}
// Parity of the completion of done[] that belongs to block g.
template <int P>
__device__ __forceinline__ uint32_t done_parity(const Shared<P>&, int g) {
  return (uint32_t)(g / Geo<P>::kStages) & 1u;
}
template <int P>
__device__ __forceinline__ uint32_t bar_final(const Shared<P>& S) { return S.bar + 8 * (Geo<P>::kNumBars - 1); }

// Bounded wait on an mbarrier phase.  Returns false when the launch has failed (here or in
// another role); the first timeout records `where`.
__device__ __forceinline__ bool wait_bar(const Args& A, volatile uint32_t* abort_flag, uint32_t bar, uint32_t parity,
                                         uint32_t where) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    if (mbar_try_sleep(bar, parity, kSleepNs)) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > A.wait_ns) {
      *abort_flag = 1u;
      atomicCAS(A.error, 0u, where);
      return false;
    }
  }
}
// Drain wait for this CTA's own copies or MMAs: bounded, but not cut short by another role's
// failure, so that nothing is still in flight into shared or tensor memory when the CTA exits.
__device__ __forceinline__ void wait_bar_drain(const Args& A, volatile uint32_t* abort_flag, uint32_t bar,
                                               uint32_t parity, uint32_t where) {
  if (mbar_try(bar, parity)) return;
  const unsigned long long t0 = gtimer();
  while (!mbar_try_sleep(bar, parity, kSleepNs)) {
    if (gtimer() - t0 > A.wait_ns) {
      *abort_flag = 1u;
      atomicCAS(A.error, 0u, where);
      return;
    }
  }
}
// Warp-uniform bounded wait: lanes leave the poll at different times, the vote reconverges the
// warp (tcgen05.ld / st are warp-aligned) and makes a timeout the whole warp's.
__device__ __forceinline__ bool warp_wait(const Args& A, volatile uint32_t* abort_flag, uint32_t bar, uint32_t parity,
                                          uint32_t where) {
  return __all_sync(0xffffffffu, wait_bar(A, abort_flag, bar, parity, where));
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

// Walks the (unit, K block) sequence of this CTA.
struct Cursor {
  int u, kb;
  Unit U;
  __device__ __forceinline__ void start(const Args& A, int n_units) {
    u = blockIdx.x;
    if (u < n_units) { U = unit_of(A, u); kb = U.kb0; }
  }
  __device__ __forceinline__ bool valid(int n_units) const { return u < n_units; }
  __device__ __forceinline__ void next(const Args& A, int n_units) {
    if (++kb >= U.kb1) {
      u += gridDim.x;
      if (u < n_units) { U = unit_of(A, u); kb = U.kb0; }
    }
  }
};

// Number of K blocks this CTA processes over all its units.
__device__ __forceinline__ int cta_blocks(const Args& A, int n_units) {
  int n = 0;
  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const Unit U = unit_of(A, u);
    n += U.kb1 - U.kb0;
  }
  return n;
}

// Warp roles: 0 = bulk-copy producer (one lane), 1 = tensor-memory owner and MMA issuer (one
// lane), 2 = none (keeps the dequantiser and epilogue groups aligned to the lane quadrants),
// 3 .. kEpiWarp0 - 1 = dequantisers (one or two sets of four), the next 8 = epilogue.  A warp may
// only touch tensor-memory lanes 32 * (warp % 4) .. +31, so each group of four covers the 128
// rows once; two dequantiser sets take alternate blocks, the two epilogue groups the two halves
// of the unit's tokens.
template <int P>
__global__ void __launch_bounds__(Geo<P>::kThreads, 1) k_tc_gemm(Args A) {
  using Gm = Geo<P>;
  extern __shared__ __align__(1024) uint8_t tc_smem[];
  __shared__ uint32_t s_tmem;
  __shared__ volatile uint32_t s_abort;
  Shared<P> S;
  S.base = (smem_u32(tc_smem) + 1023u) & ~1023u;
  S.side = S.base + Gm::kStages * Gm::kStageBytes;
  S.bar = S.side + Gm::kSide * Gm::kSideBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = A.tiles * A.tok_tiles * A.splits;

  if (threadIdx.x == 0) {
    s_abort = 0u;
    for (int s = 0; s < Gm::kStages; ++s) {
      mbar_init(bar_full(S, s), 1);
      mbar_init(bar_done(S, s), 1);
    }
    for (int b = 0; b < kBufsA; ++b) mbar_init(bar_afull(S, b), 4);
    for (int b = 0; b < kBufsD; ++b) mbar_init(bar_dempty(S, b), 8);
    for (int j = 0; j < Gm::kSide; ++j) {
      mbar_init(bar_sfull(S, j), 4);
      mbar_init(bar_sempty(S, j), 8);
    }
    mbar_init(bar_final(S), 1);
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
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: activation image + weight record per K block ----------------
      Cursor c, ahead;
      c.start(A, n_units);
      ahead.start(A, n_units);
      for (int i = 0; i < kPrefetch && ahead.valid(n_units); ++i) {
        prefetch_l2(A.recs + ((size_t)ahead.U.tile * A.kb_total + ahead.kb) * kRecBytes, kRecBytes);
        ahead.next(A, n_units);
      }
      grid_dep_wait();  // the weight records are constant; the activation image is not
      int g = 0;
      for (; c.valid(n_units) && !s_abort; c.next(A, n_units), ++g) {
        const int s = g % Gm::kStages;
        if (g >= Gm::kStages && !wait_bar(A, &s_abort, bar_done(S, s), done_parity(S, g - Gm::kStages), 1)) break;
        const uint32_t st = S.base + s * Gm::kStageBytes;
        const uint32_t fb = bar_full(S, s);
        mbar_expect_tx(fb, Gm::kStageTx);
        if (P == 1) {
          bulk_g2s(st, A.img + ((size_t)c.U.tt * A.kb_total + c.kb) * kImgBytes, kImgBytes, fb);
        } else {
          // the group's two tiles, atoms regrouped so that each K slice's hi (lo) parts of both
          // tiles form one 128-row B operand; a second tile past the image (an odd tile count)
          // repeats the first, whose rows the epilogue then does not store
          const int t0 = 2 * c.U.tt, t1 = min(t0 + 1, A.img_tiles - 1);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const uint8_t* im = A.img + ((size_t)(t ? t1 : t0) * A.kb_total + c.kb) * kImgBytes;
#pragma unroll
            for (int kh = 0; kh < 2; ++kh) {
              bulk_g2s(st + (2 * kh + t) * kAtom, im + 2 * kh * kAtom, kAtom, fb);
              bulk_g2s(st + Gm::kOffLo + (2 * kh + t) * kAtom, im + (2 * kh + 1) * kAtom, kAtom, fb);
            }
            bulk_g2s(st + Gm::kOffXs + t * kTok * 4, im + kOffXs, kTok * 4, fb);
          }
        }
        bulk_g2s(st + Gm::kOffRec, A.recs + ((size_t)c.U.tile * A.kb_total + c.kb) * kRecBytes, kRecBytes, fb);
        trace_ev(A, 0, g);
        if (ahead.valid(n_units)) {
          prefetch_l2(A.recs + ((size_t)ahead.U.tile * A.kb_total + ahead.kb) * kRecBytes, kRecBytes);
          ahead.next(A, n_units);
        }
      }
      // drain: every issued stage must have landed before the CTA may exit
      const int issued = g;
      for (int s = 0; s < Gm::kStages && s < issued; ++s) {
        const int last = issued - 1 - ((issued - 1 - s) % Gm::kStages);  // last fill of stage s
        wait_bar_drain(A, &s_abort, bar_full(S, s), (last / Gm::kStages) & 1, 2);
      }
    }
  } else if (warp == 1) {
    grid_dep_wait();
    if (lane == 0) {
      // ---------------- MMA issuer (one thread issues every MMA of the CTA) ----------------
      // Issuing from two threads that take alternate blocks was measured to corrupt an occasional
      // block, so a single thread issues all MMAs.  P = 1: one MMA (N = 128) per 16-wide K step,
      // B rows 0..63 the tokens' hi parts and rows 64..127 their lo parts (the adjacent atoms),
      // so D columns 0..63 and 64..127 accumulate q . x_hi and q . x_lo.  P = 2: two MMAs
      // (N = 128 tokens) per K step, B = the 128 tokens' hi parts, then their lo parts, both into
      // D column t.  The loop is kept short: it runs on a sub-partition shared with busy dequant
      // and epilogue warps.
      const uint32_t idesc = idesc_bf16(128);
      const int nblk = cta_blocks(A, n_units);
      const uint32_t desc_hi = (uint32_t)(sw128_desc(0) >> 32);
      const uint32_t desc_lo0 = (uint32_t)sw128_desc(S.base);
      // test only: phase 0 of the final barrier completes only after the last commit below, so
      // this wait runs out and the launch takes its error path
      if (A.expire) wait_bar(A, &s_abort, bar_final(S), 0, 13);
      for (int g = 0; g < nblk; ++g) {
        const int s = g % Gm::kStages, n = g / Gm::kStages;
        const int ba = g % kBufsA, na = g / kBufsA, bd = g % kBufsD, nd = g / kBufsD;
        // The issuer waits for the stage's bulk copies itself: the MMAs read the stage through the
        // async proxy, and the copies' completion is only guaranteed visible to them through this
        // thread's own wait on the full barrier (the dequantisers' later hand-off is not enough).
        trace_ev(A, 8, g);
        // the three inputs are normally ready long before: test all three at once (independent
        // non-blocking tests, so their latencies overlap), and take the bounded waits only if one
        // is still pending
        bool ok = mbar_test(bar_full(S, s), n & 1) & mbar_test(bar_afull(S, ba), na & 1) &
                  (mbar_test(bar_dempty(S, bd), (nd - 1) & 1) | (g < kBufsD));
        trace_ev(A, 9, g);
        if (!ok)
          ok = wait_bar(A, &s_abort, bar_full(S, s), n & 1, 3) && wait_bar(A, &s_abort, bar_afull(S, ba), na & 1, 4) &&
               (g < kBufsD || wait_bar(A, &s_abort, bar_dempty(S, bd), (nd - 1) & 1, 5));
        if (!ok) break;
        trace_ev(A, 1, g);
        tc_fence_after();
        const uint32_t dl = desc_lo0 + (uint32_t)(s * (Gm::kStageBytes >> 4));
        const uint32_t d = tmem + kDCol + bd * 128;
        const uint32_t a_t = tmem + ba * 64;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // K slice k >> 2's hi rows start 2 atoms further on, a 16-wide step is 32 bytes of a row
          const uint32_t kl = dl + (uint32_t)((((k >> 2) * 2 * kAtom) + (k & 3) * 32) >> 4);
          tc_mma_ts(d, a_t + 8 * k, ((uint64_t)desc_hi << 32) | kl, idesc, k > 0);
          if (P == 2)
            tc_mma_ts(d, a_t + 8 * k, ((uint64_t)desc_hi << 32) | (kl + (uint32_t)(Gm::kOffLo >> 4)), idesc, 1u);
        }
        trace_ev(A, 6, g);
        tc_commit(bar_done(S, s));
        trace_ev(A, 7, g);
      }
      // all issued MMAs complete before the tensor memory is released
      tc_commit(bar_final(S));
      wait_bar_drain(A, &s_abort, bar_final(S), 0, 6);
    }
  } else if (warp == 2) {
    // no role
  } else if (warp < Gm::kEpiWarp0) {
    // ---------------- dequantisers: nibbles -> bf16 codes in tensor memory ----------------
    // with two sets of four warps, set h takes blocks g with g % 2 == h, so one set's waits and
    // tensor-memory store latency overlap the other's work; warp (q, h) converts rows
    // 32q .. 32q+31 of its blocks
    const int q = warp & 3, h = (warp - 3) >> 2;
    const bool trace_warp = ((warp - 3) & 3) == 0;
    const int r = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const int sw = (r >> 1) & 3;
    const int nblk = cta_blocks(A, n_units);
    // A[b] is free once the MMAs of block g - kBufsA have completed.  The wait is on block
    // g - kFreeA: commits complete in issue order, so its completion implies that of g - kBufsA,
    // and the next phase of its done barrier is block g's own (kFreeA <= kStages), which cannot
    // complete before this warp has written A.  With fewer stages than A buffers, block
    // g - kBufsA's barrier would alias: the other set's block g - 1 reuses it and can complete
    // it again before this wait starts.
    constexpr int kFreeA = Gm::kStages < kBufsA ? Gm::kStages : kBufsA;
    for (int g = h; g < nblk; g += Gm::kDqSets) {
      const int s = g % Gm::kStages, n = g / Gm::kStages, b = g % kBufsA;
      const int j = g % Gm::kSide, nj = g / Gm::kSide;
      // side slot j is free once the epilogue has read block g - kSide
      if (!warp_wait(A, &s_abort, bar_full(S, s), n & 1, 8) ||
          (g >= kFreeA &&
           !warp_wait(A, &s_abort, bar_done(S, (g - kFreeA) % Gm::kStages), done_parity(S, g - kFreeA), 10)) ||
          (g >= Gm::kSide && !warp_wait(A, &s_abort, bar_sempty(S, j), (nj - 1) & 1, 11)))
        break;
      if (trace_warp) trace_ev(A, 2, g);
      const uint32_t st = S.base + s * Gm::kStageBytes;
      const uint32_t rec = st + Gm::kOffRec + 64 * r;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint4 c0 = lds128(rec + (uint32_t)(((2 * half) ^ sw) << 4));
        const uint4 c1 = lds128(rec + (uint32_t)(((2 * half + 1) ^ sw) << 4));
        const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        uint32_t v[32];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const uint32_t w4 = w[jj] >> 4;
          v[4 * jj + 0] = nib_pair_bf16<0>(w[jj], w4);
          v[4 * jj + 1] = nib_pair_bf16<1>(w[jj], w4);
          v[4 * jj + 2] = nib_pair_bf16<2>(w[jj], w4);
          v[4 * jj + 3] = nib_pair_bf16<3>(w[jj], w4);
        }
        tmem_st32(tmem + lane_base + b * 64 + 32 * half, v);
      }
      // scales of this row and (one warp) the unit's block sums into side slot j
      const uint32_t sd = S.side + j * Gm::kSideBytes;
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(sd + 4 * r), "r"(lds32(st + Gm::kOffRec + kNibBytes + 4 * r))
                   : "memory");
      if (q == 0) {
        if (P == 1) {
          const uint2 x2 = lds64(st + Gm::kOffXs + 8 * lane);
          asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(sd + kM * 4 + 8 * lane), "r"(x2.x), "r"(x2.y)
                       : "memory");
        } else {
          const uint4 x4 = lds128(st + Gm::kOffXs + 16 * lane);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(sd + kM * 4 + 16 * lane), "r"(x4.x),
                       "r"(x4.y), "r"(x4.z), "r"(x4.w)
                       : "memory");
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_n(bar_afull(S, b), 1);
        mbar_arrive_n(bar_sfull(S, j), 1);
      }
      if (trace_warp) trace_ev(A, 3, g);
    }
  } else {
    // ---------------- epilogue: per-block scales in fp32, unit results ----------------
    // warp (q, h): rows 32q .. 32q+31, the unit's tokens kHalf h .. kHalf h + kHalf - 1
    const int q = warp & 3, h = (warp - Gm::kEpiWarp0) >> 2;
    const int r = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    constexpr int kHalf = Gm::kUnitTok / 2;
    float acc[kHalf];
#pragma unroll
    for (int i = 0; i < kHalf; ++i) acc[i] = 0.0f;
    Cursor c;
    c.start(A, n_units);
    for (int g = 0; c.valid(n_units); c.next(A, n_units), ++g) {
      const int b = g % kBufsD, j = g % Gm::kSide, nj = g / Gm::kSide;
      if (!warp_wait(A, &s_abort, bar_done(S, g % Gm::kStages), done_parity(S, g), 7) ||
          !warp_wait(A, &s_abort, bar_sfull(S, j), nj & 1, 12))
        break;
      if (warp == Gm::kEpiWarp0) trace_ev(A, 4, g);
      tc_fence_after();
      const uint32_t sd = S.side + j * Gm::kSideBytes;
      const uint32_t sc = lds32(sd + 4 * r);
      const float step = bf16_bits_to_f32(sc & 0xFFFFu), mn = bf16_bits_to_f32(sc >> 16);
#pragma unroll
      for (int cc = 0; cc < kHalf / 16; ++cc) {
        // P = 1: token i's x_hi and x_lo products in columns i and 64 + i; P = 2: their sum in i
        uint32_t dv[16], dw[16];
        const uint32_t dcol = tmem + lane_base + kDCol + b * 128 + kHalf * h + 16 * cc;
        tmem_ld16(dcol, dv);
        if (P == 1) tmem_ld16(dcol + kTok, dw);
        tmem_wait_ld();
        if (cc == kHalf / 16 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_n(bar_dempty(S, b), 1);
        }
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const uint4 x4 = lds128(sd + kM * 4 + 4 * (kHalf * h + 16 * cc + i));
          const float xs[4] = {__uint_as_float(x4.x), __uint_as_float(x4.y), __uint_as_float(x4.z),
                               __uint_as_float(x4.w)};
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            float& a = acc[16 * cc + i + jj];
            const float dq = P == 1 ? __uint_as_float(dv[i + jj]) + __uint_as_float(dw[i + jj])
                                    : __uint_as_float(dv[i + jj]);
            a = fmaf(step, dq, fmaf(mn, xs[jj], a));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_n(bar_sempty(S, j), 1);
      if (warp == Gm::kEpiWarp0) trace_ev(A, 5, g);
      if (c.kb + 1 == c.U.kb1) {  // unit complete: store its rows
        int n = c.U.tile * kM + r;
        bool store = true;
        if (A.swiglu) {  // rows r (gate, r even) and r + 1 (up) are ffn row tile * 64 + r / 2
#pragma unroll
          for (int i = 0; i < kHalf; ++i) {
            const float up = __shfl_xor_sync(0xffffffffu, acc[i], 1);
            acc[i] = __fdividef(acc[i], 1.0f + __expf(-acc[i])) * up;
          }
          n = c.U.tile * (kM / 2) + (r >> 1);
          store = (r & 1) == 0;
        }
        const int tok0 = c.U.tt * Gm::kUnitTok + kHalf * h;
        const int nt = min(kHalf, A.T - tok0);
        float* o = A.out + (size_t)c.U.split * A.split_stride + (size_t)tok0 * A.ldo + n;
        if (store && n < A.N) {
#pragma unroll
          for (int i = 0; i < kHalf; ++i) {
            if (i < nt) *o = acc[i];
            o += A.ldo;
          }
        }
#pragma unroll
        for (int i = 0; i < kHalf; ++i) acc[i] = 0.0f;
      }
    }
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
// stride * (n % G) of a record arena with kb_total = W.K / 128 blocks per tile (G = 128,
// stride = 1, off = 0 for plain and concatenated matrices; G = 64, stride = 2, off = 0 / 1 for the
// gate / up rows of gate-up tiles, so gate row f and up row f are tile rows 2 (f % 64) and
// 2 (f % 64) + 1: adjacent lanes of one epilogue warp).
// ---------------------------------------------------------------------------------------------
__global__ void k_tc_repack(QMat W, uint8_t* __restrict__ recs, int row0, int G, int off, int stride) {
  const int kbt = W.K >> 7;
  const size_t total = (size_t)W.N * kbt * 4;  // one thread per 16-byte nibble chunk
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i & 3);
    const size_t nb = i >> 2;
    const int n = (int)(nb / kbt), kb = (int)(nb % kbt);
    const int dr = row0 + (n / G) * kM + off + stride * (n % G);
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
// Activation staging: for token row t (one CTA of 256 threads), form the GEMM input row and write
// row t of the activation image (bf16 hi / lo parts in the swizzled atom layout, and the 128-wide
// block sums of compute_x_block_sums, src/llama_engine.cpp:496-521).  The input row is
//   * x[t] (+ sum_s part[s][t], the split-K partials of the previous projection, folded into the
//     residual x, which is written back: x += proj, :1024-1025 and :1033-1034), rms-normalised
//     with gamma when given (rms_norm, :87-115); or x[t] as it is (the attention output, or the
//     SwiGLU activations silu(g) * u, :362-491, that the gate-up GEMM's epilogue wrote).
// K is a multiple of 2048; a thread handles runs of 8 consecutive elements.  Without gamma the
// grid is (tokens, K / 2048), one 2048-wide run per CTA; with gamma (tokens, 1).
// ---------------------------------------------------------------------------------------------
// kAllPlanes: all split-K planes' loads in flight at once (one round trip; more registers, so for
// steps of few rows, where latency matters more than occupancy), else three at a time.
template <bool kAllPlanes>
__global__ void __launch_bounds__(256) k_tc_stage(float* __restrict__ x, int ldx, const float* __restrict__ part,
                                                  int nsplit, size_t split_stride, const float* __restrict__ gamma,
                                                  int K, uint8_t* __restrict__ img) {
  grid_dep_begin();
  __shared__ float red[32];
  const int t = blockIdx.x;
  // runs of 8 elements per thread: j0 .. j1-1 (all K / 2048 runs when normalising, which needs
  // the whole row; otherwise gridDim.y CTAs share the row, one run each)
  const int j0 = gamma ? 0 : blockIdx.y;
  const int j1 = gamma ? K / 2048 : blockIdx.y + 1;
  const int kbt = K >> 7;
  float v[32];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j < j0 || j >= j1) continue;
    const int i0 = j * 2048 + threadIdx.x * 8;
    float e[8];
    {
      float* xp = x + (size_t)t * ldx + i0;
      const float4 a = *reinterpret_cast<const float4*>(xp), b = *reinterpret_cast<const float4*>(xp + 4);
      e[0] = a.x; e[1] = a.y; e[2] = a.z; e[3] = a.w; e[4] = b.x; e[5] = b.y; e[6] = b.z; e[7] = b.w;
      if (nsplit > 0) {
        const float* pp = part + (size_t)t * K + i0;
        float s8[8];
        {
          const float4 p0 = *reinterpret_cast<const float4*>(pp), p1 = *reinterpret_cast<const float4*>(pp + 4);
          s8[0] = p0.x; s8[1] = p0.y; s8[2] = p0.z; s8[3] = p0.w; s8[4] = p1.x; s8[5] = p1.y; s8[6] = p1.z; s8[7] = p1.w;
        }
        // planes in order
        int sp = 1;
        if (kAllPlanes && nsplit <= 8) {
          float4 q[7][2];
#pragma unroll
          for (int j = 0; j < 7; ++j) {
            if (1 + j < nsplit) {
              q[j][0] = *reinterpret_cast<const float4*>(pp + (1 + j) * split_stride);
              q[j][1] = *reinterpret_cast<const float4*>(pp + (1 + j) * split_stride + 4);
            }
          }
#pragma unroll
          for (int j = 0; j < 7; ++j) {
            if (1 + j < nsplit) {
              s8[0] += q[j][0].x; s8[1] += q[j][0].y; s8[2] += q[j][0].z; s8[3] += q[j][0].w;
              s8[4] += q[j][1].x; s8[5] += q[j][1].y; s8[6] += q[j][1].z; s8[7] += q[j][1].w;
            }
          }
          sp = nsplit;
        }
        for (; sp + 2 < nsplit; sp += 3) {  // three planes' loads in flight at a time
          float4 q[3][2];
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            q[j][0] = *reinterpret_cast<const float4*>(pp + (sp + j) * split_stride);
            q[j][1] = *reinterpret_cast<const float4*>(pp + (sp + j) * split_stride + 4);
          }
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            s8[0] += q[j][0].x; s8[1] += q[j][0].y; s8[2] += q[j][0].z; s8[3] += q[j][0].w;
            s8[4] += q[j][1].x; s8[5] += q[j][1].y; s8[6] += q[j][1].z; s8[7] += q[j][1].w;
          }
        }
        for (; sp < nsplit; ++sp) {
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
      if (j < j0 || j >= j1) continue;
      const int i0 = j * 2048 + threadIdx.x * 8;
#pragma unroll
      for (int k = 0; k < 8; ++k) v[j * 8 + k] = __fmul_rn(__fmul_rn(v[j * 8 + k], gamma[i0 + k]), inv);
    }
  }
  const int tt = t / kTok, tr = t % kTok;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j < j0 || j >= j1) continue;
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
    const size_t o = (size_t)atom * 2 * kAtom + tr * 128 + ((c ^ (tr & 7)) << 4);
    *reinterpret_cast<uint4*>(im + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(im + kAtom + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    // 16 threads cover one 128-block
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o2);
    if ((threadIdx.x & 15) == 0) reinterpret_cast<float*>(im + kOffXs)[tr] = bs;
  }
}

// ---------------------------------------------------------------------------------------------
// RoPE and KV append for token row t of a q | k | v GEMM output (src/llama_engine.cpp:953-956,
// apply_rope :120-151 with the host-built table), summing its nsplit split-K planes first:
// rotated q to q_out[t], rotated k and v into the cache row (slot[t], pos[t]).  One CTA of 256
// threads per token row; a thread rotates kRopePer pairs at a time with all their loads issued
// before any store, then copies v elements.
// ---------------------------------------------------------------------------------------------
// Sum of the nsplit planes in plane order; four loads in flight at a time.
__device__ __forceinline__ float sum_planes(const float* p, int nsplit, size_t stride) {
  float v = p[0];
  int s = 1;
  for (; s + 3 < nsplit; s += 4) {
    const float a = p[s * stride], b = p[(s + 1) * stride], c = p[(s + 2) * stride], d = p[(s + 3) * stride];
    v += a;
    v += b;
    v += c;
    v += d;
  }
  for (; s < nsplit; ++s) v += p[s * stride];
  return v;
}
constexpr int kRopePer = 5;  // (q_dim + kv_dim) / 2 = 1280 pairs per 2048 of dim: 5 per thread
__global__ void __launch_bounds__(256) k_rope_append(const float* __restrict__ qkv, int nsplit, size_t split_stride,
                                                     int q_dim, int kv_dim, const int32_t* __restrict__ pos,
                                                     const int32_t* __restrict__ slot, const float* __restrict__ rope_cos,
                                                     const float* __restrict__ rope_sin, float* __restrict__ q_out,
                                                     float* __restrict__ kc, float* __restrict__ vc, size_t slot_stride) {
  grid_dep_begin();
  const int t = blockIdx.x;
  const int p = pos[t];
  const float* row = qkv + (size_t)t * (q_dim + 2 * kv_dim);
  const size_t cache = (size_t)slot[t] * slot_stride + (size_t)p * kv_dim;
  const int npairs = (q_dim + kv_dim) / 2;  // rotated pairs (i, i + 32) of the q and k heads
  for (int j0 = threadIdx.x; j0 < npairs; j0 += kRopePer * 256) {
    float r0[kRopePer], r1[kRopePer], c[kRopePer], sn[kRopePer];
#pragma unroll
    for (int k = 0; k < kRopePer; ++k) {
      const int j = j0 + 256 * k;
      if (j < npairs) {
        const int i = j & 31, base = (j >> 5) * LE_HEAD_DIM + i;  // q heads first, then k heads
        if (nsplit == 1) {
          r0[k] = row[base];
          r1[k] = row[base + 32];
        } else {
          r0[k] = sum_planes(row + base, nsplit, split_stride);
          r1[k] = sum_planes(row + base + 32, nsplit, split_stride);
        }
        c[k] = rope_cos[p * 32 + i];
        sn[k] = rope_sin[p * 32 + i];
      }
    }
#pragma unroll
    for (int k = 0; k < kRopePer; ++k) {
      const int j = j0 + 256 * k;
      if (j < npairs) {
        const int base = (j >> 5) * LE_HEAD_DIM + (j & 31);
        const float o0 = __fsub_rn(__fmul_rn(r0[k], c[k]), __fmul_rn(r1[k], sn[k]));
        const float o1 = __fadd_rn(__fmul_rn(r0[k], sn[k]), __fmul_rn(r1[k], c[k]));
        if (base < q_dim) {
          q_out[(size_t)t * q_dim + base] = o0;
          q_out[(size_t)t * q_dim + base + 32] = o1;
        } else {
          kc[cache + base - q_dim] = o0;
          kc[cache + base - q_dim + 32] = o1;
        }
      }
    }
  }
  const float* vrow = row + q_dim + kv_dim;
  for (int e0 = threadIdx.x; e0 < kv_dim; e0 += 2 * 256) {
    const int e1 = e0 + 256;
    const float v0 = sum_planes(vrow + e0, nsplit, split_stride);
    const float v1 = e1 < kv_dim ? sum_planes(vrow + e1, nsplit, split_stride) : 0.0f;
    vc[cache + e0] = v0;
    if (e1 < kv_dim) vc[cache + e1] = v1;
  }
}

}  // namespace tc
}  // namespace le
