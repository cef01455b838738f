// Persistent token-step kernel for batch-1 decode (sm_100a).
//
// One cooperative launch runs whole token steps (src/llama_engine.cpp:935-1042 and the greedy
// sampler :784-792): one CTA of 16 warps per SM.  The CTA's weight records stream from HBM into
// a 10-slot shared-memory ring with cp.async.bulk (TMA bulk copies) and mbarriers: the ring is
// filled at start, and the warps that finish a record immediately issue the copy of the record
// ten positions later into the freed slot, so the weight stream runs ahead across phases and
// layers (weights never depend on activations).  Phase by phase the warps stage the phase's
// input vector as MMA digit fragments (rms-norm fused where the reference normalises) and reduce
// their records on the integer tensor-core path (mma_gemv.cuh).
// Phases of layer l: QKV rows -> attention per head (RoPE, KV append, softmax, PV) -> o-proj
// rows (+ residual) -> gate/up rows (SiLU * up) -> down rows (+ residual); then lm_head rows with
// a fused greedy argmax.  Every phase's work is split statically over the CTAs by a host-built
// schedule.
//
// Hand-offs between phases are self-validating: every activation element (x, q|k|v, attention
// output, SwiGLU output) is one 64-bit word, fp32 value in the low half and a phase tag in the
// high half, written with one 64-bit store and read with 64-bit relaxed loads, so a staging load
// is its own readiness check (no fences, counters or polls on the data path).  The tag of
// (token step s, layer l, phase p) is unique over a launch and its neighbours.  Each element has
// exactly one writer per phase, and the dependency chain guarantees that no element is
// overwritten before every reader of its previous value has read it.
//
// All waits are bounded in time (PArgs::wait_ns); on timeout a global error word is set, every
// later wait returns at once, the CTA issues no further copies and waits for the ones in flight,
// and the launch drains, so the host sees an error, never a hang.
//
// Record format (built at load time from the LLM4S128 matrices): 16 rows x 16 blocks
// (2048 columns) of one matrix, 17408 bytes:
//   [0, 16384): block j = 0..15 takes 1024 bytes: for lane L = 0..31 (g = L/4, t = L%4), the 16
//               bytes of row g at block bytes [16t, 16t+16) at j*1024 + L*16, and the 16 bytes of
//               row g+8 at j*1024 + 512 + L*16 (the MMA A fragments, conflict-free 16-byte loads);
//   [16384, 17408): for block j, row r = 0..15: u32 = step_bf16 | min_bf16 << 16.
#pragma once

#include "mma_gemv.cuh"

namespace le {

constexpr int kRecBytes = 17408;
constexpr int kRecNibBytes = 16384;
constexpr int kPConsumerWarps = 16;
constexpr int kPThreads = 32 * kPConsumerWarps;
constexpr int kRingSlots = 10;
constexpr int kMiscFloats = 2304;          // attention scratch (q, k, v, reductions, 32x64 partials),
                                           // or the row partials of a segment's work units
constexpr int kMaxUnits = kMiscFloats / 16;  // work units per segment
constexpr int kImageBytes = 32768 + 1024;  // digit fragments for K <= 8192, or attention scores
constexpr unsigned long long kWaitNs = 2000000000ull;  // default bound on every wait (2 s)
constexpr unsigned kPollNs = 20;  // pause between polls of tagged activations
constexpr int kTraceCap = 1024;

enum PKind : uint16_t { PK_QKV = 0, PK_ATTN, PK_O, PK_GATEUP, PK_DOWN, PK_LMHEAD };
// phase tags of the activation hand-offs
enum PTag : uint32_t { TG_XIN = 0, TG_QKV = 1, TG_ATTN = 2, TG_XO = 3, TG_ACT = 4 };

// Schedule entries are packed small: each CTA copies its whole schedule into shared memory at
// launch, so no descriptor load sits on the critical path.
struct PItem {
  uint8_t kind, nrec;
  uint16_t layer;
  uint16_t tile;      // row tile (16 rows) within the phase's row space; head index for PK_ATTN
  uint16_t rec;       // first record of the item in the CTA's per-token record stream
};

struct PSeg {
  uint8_t kind;
  uint8_t split;      // work units per record (1, 2, 4, 8 or 16 block ranges)
  uint16_t layer;
  uint16_t item_begin, item_end;
};

constexpr int kMaxRecs = 512;   // per CTA and token
constexpr int kMaxItems = 512;
constexpr int kMaxSegs = 128;
constexpr int kSchedBytes = kMaxRecs * 4 + kMaxItems * 8 + kMaxSegs * 8;

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
  uint32_t lm_ctr;     // CTAs done with the lm_head (monotonic, generate-mode token feedback)
  uint32_t never;      // never written: the target of the test-only expiring wait
  uint32_t pad;
  unsigned long long key[3];  // packed greedy candidates, by lm step modulo 3
};

struct PArgs {
  const uint8_t* arena;           // repacked records
  const PCtaSched* sched;
  const PSeg* segs;
  const PItem* items;
  const uint32_t* recs;           // record indices into `arena` (byte offset = index * kRecBytes)
  const float* norms;             // [2*layers + 1][dim]: in_norm[l], post_norm[l] ..., final_norm
  const float* rope_cos;
  const float* rope_sin;
  unsigned long long* x;    // [dim]            tagged
  unsigned long long* qkv;  // [dim + 2 kv_dim] tagged
  unsigned long long* attn; // [dim]            tagged
  unsigned long long* act;  // [ffn]            tagged
  float* logits;    // [vocab]
  float* kcache;    // slot 0: [layers][max_seq][kv_dim]
  float* vcache;
  PCtrl* ctrl;
  int32_t* token_log;
  int32_t* am_result;
  unsigned long long lm_rec_base;  // record offset of lm_head tile 0 (embedding lookup)
  unsigned long long wait_ns;      // bound on every wait
  int layers, dim, ffn, vocab, heads, kv_heads, max_seq;
  int n_lm_ctas;
  int n_tokens, do_logits;
  int token0, pos0;  // the first step's token id and position (later steps feed back the greedy id)
  // optional mapped host words, written by the last CTA to finish: error, err_where, greedy id
  // (with logits), then `seq` (after a system-scope fence) so that the host can wait on it
  uint32_t* host_done;
  uint32_t seq;
  int expire_where;  // test only: nonzero makes CTA 0 wait on PCtrl::never with this code
  unsigned long long* trace;  // optional: per CTA kTraceCap (time, tag) pairs, first token only
};

__device__ __forceinline__ uint32_t phase_tag(uint32_t s, int layers, int l, uint32_t p) {
  return ((s * (uint32_t)(layers + 1) + (uint32_t)l) << 3) + p + 1u;
}

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
__device__ __forceinline__ void mbar_arrive_n(uint32_t a, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(n) : "memory");
}
// Non-blocking test of phase `parity` (acquire, CTA scope).
__device__ __forceinline__ bool mbar_test(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a thread whose phase is pending sleeps (up to hint_ns) until
// the phase completes instead of returning at once, so waiting warps take no issue slots.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t a, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(a), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
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
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) { return __uint_as_float(lds32(a)); }
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ld_tag2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tag(const unsigned long long* p) {
  unsigned long long a;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}
__device__ __forceinline__ void st_tag(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ float tag_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ uint32_t tag_of(unsigned long long w) { return (uint32_t)(w >> 32); }

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
__device__ bool wait_counter(const PArgs& A, const uint32_t* p, uint32_t target, uint32_t where) {
  if (reached(ld_acquire(p), target)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    if (failed(A)) return false;
    if (reached(ld_acquire(p), target)) return true;
    if (gtimer() - t0 > A.wait_ns) { fail(A, where); return false; }
    __nanosleep(40);
  }
}

__device__ bool wait_mbar(const PArgs& A, uint32_t bar, uint32_t parity, uint32_t where) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (failed(A)) return false;
    if (gtimer() - t0 > A.wait_ns) { fail(A, where); return false; }
  }
}

// Drain wait for a copy this CTA issued: bounded, but not cut short by another wait's failure,
// so that no copy is still in flight into shared memory when the CTA exits.
__device__ void wait_mbar_drain(const PArgs& A, uint32_t bar, uint32_t parity, uint32_t where) {
  if (mbar_try(bar, parity)) return;
  const unsigned long long t0 = gtimer();
  while (!mbar_try(bar, parity)) {
    if (gtimer() - t0 > A.wait_ns) { fail(A, where); return; }
  }
}

// Waits until ring slot `slot` has been issued record q (bounded).
__device__ __forceinline__ bool wait_slot(const PArgs& A, volatile int* slot_rec, uint32_t slot, uint32_t q,
                                          uint32_t where) {
  if (slot_rec[slot] == (int)q) return true;
  const unsigned long long t0 = gtimer();
  while (slot_rec[slot] != (int)q) {
    if (failed(A)) return false;
    if (gtimer() - t0 > A.wait_ns) { fail(A, where); return false; }
    __nanosleep(20);
  }
  return true;
}

// Loads N2 pairs of tagged words starting at p until every tag equals `tag` (bounded).
template <int N2>
__device__ __forceinline__ void ld_tagged(const PArgs& A, const unsigned long long* p, uint32_t tag, float* out,
                                          uint32_t where) {
  unsigned long long w[2 * N2];
#pragma unroll
  for (int i = 0; i < N2; ++i) ld_tag2(p + 2 * i, w[2 * i], w[2 * i + 1]);
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 2 * N2; ++i) ok &= tag_of(w[i]) == tag;
  if (!ok) {
    const unsigned long long t0 = gtimer();
    while (true) {
#pragma unroll
      for (int i = 0; i < N2; ++i) ld_tag2(p + 2 * i, w[2 * i], w[2 * i + 1]);
      ok = true;
#pragma unroll
      for (int i = 0; i < 2 * N2; ++i) ok &= tag_of(w[i]) == tag;
      if (ok || failed(A)) break;
      if (gtimer() - t0 > A.wait_ns) { fail(A, where); break; }
      __nanosleep(kPollNs);
    }
  }
#pragma unroll
  for (int i = 0; i < 2 * N2; ++i) out[i] = tag_val(w[i]);
}

// Two groups of 8 tagged words (p and q) loaded together, so both take one round trip.
__device__ __forceinline__ void ld_tagged2x(const PArgs& A, const unsigned long long* p, const unsigned long long* q,
                                            uint32_t tag, float* out0, float* out1, uint32_t where) {
  unsigned long long w[16];
  auto load = [&]() {
#pragma unroll
    for (int i = 0; i < 4; ++i) ld_tag2(p + 2 * i, w[2 * i], w[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) ld_tag2(q + 2 * i, w[8 + 2 * i], w[8 + 2 * i + 1]);
  };
  auto all_ok = [&]() {
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 16; ++i) ok &= tag_of(w[i]) == tag;
    return ok;
  };
  load();
  if (!all_ok()) {
    const unsigned long long t0 = gtimer();
    while (true) {
      load();
      if (all_ok() || failed(A)) break;
      if (gtimer() - t0 > A.wait_ns) { fail(A, where); break; }
      __nanosleep(kPollNs);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    out0[i] = tag_val(w[i]);
    out1[i] = tag_val(w[8 + i]);
  }
}

__device__ __forceinline__ float ld_tagged1(const PArgs& A, const unsigned long long* p, uint32_t tag, uint32_t where) {
  unsigned long long w = ld_tag(p);
  if (tag_of(w) != tag) {
    const unsigned long long t0 = gtimer();
    while (true) {
      w = ld_tag(p);
      if (tag_of(w) == tag || failed(A)) break;
      if (gtimer() - t0 > A.wait_ns) { fail(A, where); break; }
      __nanosleep(kPollNs);
    }
  }
  return tag_val(w);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(~(uint32_t)idx);
}

// ---------------------------------------------------------------------------------------------
// Staging: the CTA turns an input vector of K elements into MX = 1 digit fragments
//   bfrag[(b*4 + i)*16 + p*4 + t] = (b0, b1) for digit plane p, MMA i, quad lane t of block b,
// plus block sums and scales.  8-element group q covers elements 8q..8q+7 = block q/16,
// (t, i) = ((q%16)/4, (q%16)%4); thread `tid` owns groups q = tid + 512*r (q < K/8).
// ---------------------------------------------------------------------------------------------
struct Stage {
  uint2* bfrag;
  float* bsum;
  float* escl;
  float* red;  // 32 floats
};

// Digits of one group.  The MMA's A operand is the raw nibble byte r = q_even + 16 q_odd for the
// low K-half of each fragment word and the high nibble q_odd for the high K-half, so the B
// operand carries y = x_even for the first and z = x_odd - 16 x_even for the second:
//   r * y + q_odd * z = q_even x_even + q_odd x_odd.
__device__ __forceinline__ void stage_group(const float (&x)[8], int q, const Stage& S) {
  const int b = q >> 4, ti = q & 15, t = ti >> 2, i = ti & 3;
  float v[8];
  float s = 0.0f, a = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    s += x[e] + x[e + 1];
    v[e] = x[e];
    v[e + 1] = fmaf(-16.0f, x[e], x[e + 1]);
    a = fmaxf(a, fmaxf(fabsf(v[e]), fabsf(v[e + 1])));
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
    int X = __float2int_rn(v[k] * up);
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

// rms-norm staging of a 2048-wide tagged activation: out = x * g * inv (rms_norm, :87-115).
// Threads 0..255 own one group each.
__device__ __forceinline__ void stage_norm2048_vals(const float (&xv)[8], const float4 (&gm)[2], const Stage& S) {
  const int tid = threadIdx.x;
  float ss = 0.0f;
  if (tid < 256) {
#pragma unroll
    for (int k = 0; k < 8; ++k) ss = fmaf(xv[k], xv[k], ss);
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) S.red[tid >> 5] = ss;
  consumer_sync();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kPConsumerWarps; ++w) tot += S.red[w];
  const float inv = 1.0f / sqrtf(tot / 2048.0f + 1e-5f);
  if (tid < 256) {
    const float gv[8] = {gm[0].x, gm[0].y, gm[0].z, gm[0].w, gm[1].x, gm[1].y, gm[1].z, gm[1].w};
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(__fmul_rn(xv[k], gv[k]), inv);
    stage_group(v, tid, S);
  }
  consumer_sync();
}

__device__ __forceinline__ void load_gamma(const float* gamma, float4 (&gm)[2]) {
  const int i = threadIdx.x & 255;  // threads >= 256 load a duplicate they never use
  gm[0] = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * i);
  gm[1] = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * i + 1);
}

__device__ __forceinline__ void stage_norm2048(const PArgs& A, const unsigned long long* x, uint32_t tag,
                                               const float* gamma, const Stage& S, uint32_t where) {
  float4 gm[2];
  load_gamma(gamma, gm);  // independent of the dependency: issued first
  float xv[8];
  if (threadIdx.x < 256) ld_tagged<4>(A, x + 8 * threadIdx.x, tag, xv, where);
  stage_norm2048_vals(xv, gm, S);
}

// plain staging of a tagged activation of K = 2048, 4096 or 8192 elements
__device__ __forceinline__ void stage_plain(const PArgs& A, const unsigned long long* x, int K, uint32_t tag,
                                            const Stage& S, uint32_t where) {
  const int tid = threadIdx.x;
  const int ngroups = K / 8;
  float v0[8], v1[8];
  if (tid + 512 < ngroups) ld_tagged2x(A, x + 8 * tid, x + 8 * (tid + 512), tag, v0, v1, where);
  else if (tid < ngroups) ld_tagged<4>(A, x + 8 * tid, tag, v0, where);
  if (tid < ngroups) stage_group(v0, tid, S);
  if (tid + 512 < ngroups) stage_group(v1, tid + 512, S);
  consumer_sync();
}

// ---------------------------------------------------------------------------------------------
// Blocks [j0, j0 + NBLK) of one record on the MMA path (blocks kq*16 + j of the staged input).
// MMAs i = 0,1 and 2,3 chain through two accumulators; their int32 sums are exact.  Every lane
// folds its digit planes pairwise (planes 0+1 on lanes t = 0, 2; planes 2+3 on t = 1, 3), so
// one shuffle per row brings the high planes to the owner lane t == 0.
// Lanes with t == 0 return the partial sums of rows g (p0) and g+8 (p1).
// ---------------------------------------------------------------------------------------------
template <int NB>  // NB <= 4 blocks: the three passes over one chunk
__device__ __forceinline__ void record_chunk(uint32_t r_nib, uint32_t r_sc, uint32_t s_bf, uint32_t s_es,
                                             uint32_t s_bs, int kq, int j0, float& a0, float& a1) {
  const int lane = threadIdx.x & 31, t = lane & 3;
  const bool bl = lane < 16;
  // pass 1: the MMAs of the chunk's blocks (independent across blocks)
  int xg[NB], xh[NB];
#pragma unroll
  for (int jj = 0; jj < NB; ++jj) {
    const int j = j0 + jj, b = kq * 16 + j;
    const uint4 wa = lds128(r_nib + 1024u * j);
    const uint4 wb = lds128(r_nib + 1024u * j + 512u);
    const uint32_t bfa = s_bf + 512u * b;
    // lanes 16..31 hold the zero columns 4..7 of B: only the low half-warp reads shared memory
    uint2 b0 = make_uint2(0u, 0u), b1 = b0, b2 = b0, b3 = b0;
    if (bl) {
      b0 = lds64(bfa);
      b1 = lds64(bfa + 128u);
      b2 = lds64(bfa + 256u);
      b3 = lds64(bfa + 384u);
    }
    int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
    // low K-half: raw bytes (q_even + 16 q_odd); high K-half: q_odd (see stage_group)
    mma_u8s8(c0, wa.x, wb.x, (wa.x >> 4) & 0x0F0F0F0Fu, (wb.x >> 4) & 0x0F0F0F0Fu, b0.x, b0.y);
    mma_u8s8(c1, wa.z, wb.z, (wa.z >> 4) & 0x0F0F0F0Fu, (wb.z >> 4) & 0x0F0F0F0Fu, b2.x, b2.y);
    mma_u8s8(c0, wa.y, wb.y, (wa.y >> 4) & 0x0F0F0F0Fu, (wb.y >> 4) & 0x0F0F0F0Fu, b1.x, b1.y);
    mma_u8s8(c1, wa.w, wb.w, (wa.w >> 4) & 0x0F0F0F0Fu, (wb.w >> 4) & 0x0F0F0F0Fu, b3.x, b3.y);
    // planes (2t, 2t+1) of rows g (e = 0, 1) and g+8 (e = 2, 3); fold pairwise: X = P_even + 256 P_odd
    // (|P| <= 4 MMAs * (16*255 + 16*15) * 128 < 2.3e6, so |X| < 6e8 fits int32)
    xg[jj] = (c0[0] + c1[0]) + (c0[1] + c1[1]) * 256;
    xh[jj] = (c0[2] + c1[2]) + (c0[3] + c1[3]) * 256;
  }
  // pass 2: bring the high planes (lanes t = 1, 3) to the owner lanes
  int hg[NB], hh[NB];
#pragma unroll
  for (int jj = 0; jj < NB; ++jj) {
    hg[jj] = __shfl_xor_sync(0xffffffffu, xg[jj], 1);
    hh[jj] = __shfl_xor_sync(0xffffffffu, xh[jj], 1);
  }
  // pass 3: per-block scaling on the owner lanes
  if (t == 0) {
#pragma unroll
    for (int jj = 0; jj < NB; ++jj) {
      const int j = j0 + jj, b = kq * 16 + j;
      const uint32_t s0 = lds32(r_sc + 64u * j), s1 = lds32(r_sc + 64u * j + 32u);
      const float es = ldsf(s_es + 4u * b), xsb = ldsf(s_bs + 4u * b);
      const float v0 = fmaf((float)hg[jj], 65536.0f, (float)xg[jj]);
      const float v1 = fmaf((float)hh[jj], 65536.0f, (float)xh[jj]);
      a0 += fmaf(__uint_as_float(s0 << 16) * es, v0, __uint_as_float(s0 & 0xFFFF0000u) * xsb);
      a1 += fmaf(__uint_as_float(s1 << 16) * es, v1, __uint_as_float(s1 & 0xFFFF0000u) * xsb);
    }
  }
}

// Blocks [j0, j0 + NBLK) of one record; lanes with t == 0 return rows g (p0) and g+8 (p1).
template <int NBLK>
__device__ __forceinline__ void record_part(const uint8_t* rec, int kq, int j0, const Stage& S, float& p0, float& p1) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  // explicit shared-space addressing: ring record, digit fragments, block scales
  const uint32_t r_nib = smem_u32(rec) + 16u * lane;
  const uint32_t r_sc = smem_u32(rec) + kRecNibBytes + 4u * g;
  const uint32_t s_bf = smem_u32(S.bfrag) + 8u * (lane & 15);
  const uint32_t s_es = smem_u32(S.escl), s_bs = smem_u32(S.bsum);
  float a0 = 0.f, a1 = 0.f;
  constexpr int NB = NBLK < 4 ? NBLK : 4;
#pragma unroll
  for (int c = 0; c < NBLK; c += NB) record_chunk<NB>(r_nib, r_sc, s_bf, s_es, s_bs, kq, j0 + c, a0, a1);
  p0 = a0;
  p1 = a1;
}

__device__ __forceinline__ void record_blocks(int F, const uint8_t* rec, int kq, int mi, const Stage& S, float& p0,
                                              float& p1) {
  switch (F) {
    case 2: record_part<8>(rec, kq, 8 * mi, S, p0, p1); break;
    case 4: record_part<4>(rec, kq, 4 * mi, S, p0, p1); break;
    case 8: record_part<2>(rec, kq, 2 * mi, S, p0, p1); break;
    default: record_part<1>(rec, kq, mi, S, p0, p1); break;
  }
}

// Trace entry: (%globaltimer ns or `value`, tag | low 32 bits of the SM clock << 32).  The clock
// gives cycle-exact intervals within a CTA; the global timer orders events across CTAs.
template <bool kTrace>
__device__ __forceinline__ void trace_mark(const PArgs& A, int& n, int tok, uint32_t tag,
                                           unsigned long long value = 0ull) {
  if (kTrace && A.trace != nullptr && tok == 0 && n < kTraceCap) {
    unsigned long long* tr = A.trace + ((size_t)blockIdx.x * kTraceCap + n) * 2;
    tr[0] = value ? value : gtimer();
    tr[1] = (unsigned long long)tag | ((unsigned long long)(uint32_t)clock64() << 32);
    ++n;
  }
}

// ---------------------------------------------------------------------------------------------
// Attention of one head on the CTA (src/llama_engine.cpp:953-1021): RoPE from the table, KV
// append at pos (by the first q head of each kv group), softmax over 0..pos, PV.
// Flash-decoding inside the CTA: warp w takes positions base + w + 16 i (i < kAttnP) of each
// 64-position chunk, lane d holds dims 2d and 2d+1; every warp keeps a running max, sum and
// output row, and the 16 warps are merged at the end.  The cached K and V rows do not depend on
// this step, so before the wait for q, k and v the first chunk's rows are loaded into registers
// and the second chunk's into shared memory (cp.async); later chunks are prefetched into L2.
// ---------------------------------------------------------------------------------------------
constexpr int kAttnP = 4;                           // positions per warp per chunk
constexpr int kAttnChunk = kAttnP * kPConsumerWarps;
// the second chunk is staged in the image region as [row][K 64 | V 64] floats
static_assert(kAttnChunk * 128 * 4 <= kImageBytes, "second attention chunk must fit the image region");

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <bool kTrace>
__device__ void attention_head(const PArgs& A, int l, int h, int pos, uint32_t s, float* sm, float* img, int& ntr,
                               int tok) {
  const bool fine = kTrace && threadIdx.x == 0 && (l == 1 || l == 2);
  const uint32_t ftag = ((uint32_t)PK_ATTN << 8) | (uint32_t)l;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  constexpr int NT = kPThreads;
  const int group = A.heads / A.kv_heads, kvh = h / group;
  const int kv_dim = A.kv_heads * LE_HEAD_DIM, q_dim = A.heads * LE_HEAD_DIM;
  float* sq = sm;           // 64: q after RoPE
  float* sk = sm + 64;      // 64: k after RoPE
  float* sv = sm + 128;     // 64
  float* raw = sm + 192;    // 192: q, k, v as loaded
  float* wm = sm + 384;     // 16: per-warp running max
  float* wl = sm + 400;     // 16: per-warp sum
  float* wacc = sm + 448;   // 16 x 64: per-warp output rows
  const float* kc = A.kcache + (size_t)l * A.max_seq * kv_dim + kvh * LE_HEAD_DIM;
  const float* vc = A.vcache + (size_t)l * A.max_seq * kv_dim + kvh * LE_HEAD_DIM;
  const uint32_t tq = phase_tag(s, A.layers, l, TG_QKV);

  float2 kr[kAttnP], vr[kAttnP];
  auto load_chunk = [&](int base) {
#pragma unroll
    for (int i = 0; i < kAttnP; ++i) {
      const int t = base + w + kPConsumerWarps * i;
      if (t < pos) {
        kr[i] = __ldcg(reinterpret_cast<const float2*>(kc + (size_t)t * kv_dim) + lane);
        vr[i] = __ldcg(reinterpret_cast<const float2*>(vc + (size_t)t * kv_dim) + lane);
      }
    }
  };
  load_chunk(0);
  // second chunk: rows [kAttnChunk, 2 kAttnChunk) as [row][K 64 | V 64] floats in `img`
  const int c1 = min(pos, 2 * kAttnChunk) - kAttnChunk;
  for (int pc = tid; pc < c1 * 32; pc += NT) {
    const int r = pc >> 5, part = pc & 31;  // parts 0..15: K, 16..31: V (16 bytes each)
    const float* src = (part < 16 ? kc : vc) + (size_t)(kAttnChunk + r) * kv_dim + (part & 15) * 4;
    cp_async16_s(smem_u32(img + r * 128 + (part & 16) * 4 + (part & 15) * 4), src);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // rows of later chunks: into L2 meanwhile
  for (int t = 2 * kAttnChunk + tid; t < pos; t += NT) {
    prefetch_l2(kc + (size_t)t * kv_dim, 256);
    prefetch_l2(vc + (size_t)t * kv_dim, 256);
  }
  // q, k, v of this step: one 16-byte tagged load (two elements) per thread
  if (tid < 96) {
    const unsigned long long* src = tid < 32   ? A.qkv + h * LE_HEAD_DIM + 2 * tid
                                    : tid < 64 ? A.qkv + q_dim + kvh * LE_HEAD_DIM + 2 * (tid - 32)
                                               : A.qkv + q_dim + kv_dim + kvh * LE_HEAD_DIM + 2 * (tid - 64);
    float v2[2];
    ld_tagged<1>(A, src, tq, v2, 100 + l);
    raw[2 * tid] = v2[0];
    raw[2 * tid + 1] = v2[1];
  }
  consumer_sync();
  if (tid < 64) {  // RoPE of q (tid < 32) and k: pairs (i, i + 32)
    const int i = tid & 31;
    const float* r = raw + (tid < 32 ? 0 : 64);
    float* o = tid < 32 ? sq : sk;
    const float c = A.rope_cos[pos * 32 + i], sn = A.rope_sin[pos * 32 + i];
    const float r0 = r[i], r1 = r[i + 32];
    o[i] = __fsub_rn(__fmul_rn(r0, c), __fmul_rn(r1, sn));
    o[i + 32] = __fadd_rn(__fmul_rn(r0, sn), __fmul_rn(r1, c));
  } else if (tid < 128) {
    sv[tid - 64] = raw[128 + tid - 64];
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  consumer_sync();
  if (fine) trace_mark<kTrace>(A, ntr, tok, ftag | 0xA0000u);
  // KV append by the last two warps; their fence orders the rows before everything this CTA
  // publishes after its next barrier
  if (h % group == 0 && tid >= NT - 64) {
    const int i = tid - (NT - 64);
    A.kcache[(size_t)l * A.max_seq * kv_dim + (size_t)pos * kv_dim + kvh * LE_HEAD_DIM + i] = sk[i];
    A.vcache[(size_t)l * A.max_seq * kv_dim + (size_t)pos * kv_dim + kvh * LE_HEAD_DIM + i] = sv[i];
    __threadfence();
  }
  const float2 q2 = reinterpret_cast<const float2*>(sq)[lane];
  const float2 kcur = reinterpret_cast<const float2*>(sk)[lane];
  const float2 vcur = reinterpret_cast<const float2*>(sv)[lane];
  float m = -INFINITY, lsum = 0.0f;
  float2 acc = make_float2(0.0f, 0.0f);
  for (int base = 0; base <= pos; base += kAttnChunk) {
    const bool from_img = base == kAttnChunk;
    if (base >= 2 * kAttnChunk) load_chunk(base);
    float sc[kAttnP];
    float cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < kAttnP; ++i) {
      const int t = base + w + kPConsumerWarps * i;
      const float2 kk = t >= pos   ? kcur
                        : from_img ? reinterpret_cast<const float2*>(img + (t - base) * 128)[lane]
                                   : kr[i];
      const float d = warp_allsum(fmaf(q2.x, kk.x, q2.y * kk.y));
      sc[i] = t <= pos ? d * 0.125f : -INFINITY;
      cm = fmaxf(cm, sc[i]);
    }
    if (cm == -INFINITY) continue;  // no position of this chunk on this warp (warp-uniform)
    const float mn = fmaxf(m, cm);
    const float r = expf(m - mn);
    lsum *= r;
    acc.x *= r;
    acc.y *= r;
#pragma unroll
    for (int i = 0; i < kAttnP; ++i) {
      const int t = base + w + kPConsumerWarps * i;
      if (t <= pos) {
        const float e = expf(sc[i] - mn);
        const float2 vv = t >= pos   ? vcur
                          : from_img ? reinterpret_cast<const float2*>(img + (t - base) * 128 + 64)[lane]
                                     : vr[i];
        lsum += e;
        acc.x = fmaf(e, vv.x, acc.x);
        acc.y = fmaf(e, vv.y, acc.y);
      }
    }
    m = mn;
  }
  if (fine) trace_mark<kTrace>(A, ntr, tok, ftag | 0xB0000u);
  // merge of the 16 warps: every warp rescales its own (sum, output row) to the common maximum
  // in registers, then 64 threads add the 16 rescaled rows as a tree
  if (lane == 0) wm[w] = m;
  consumer_sync();
  float M = wm[0];
#pragma unroll
  for (int v = 1; v < kPConsumerWarps; ++v) M = fmaxf(M, wm[v]);
  const float f = m == -INFINITY ? 0.0f : expf(m - M);  // a warp without positions adds nothing
  reinterpret_cast<float2*>(wacc + w * 64)[lane] = make_float2(acc.x * f, acc.y * f);
  if (lane == 0) wl[w] = lsum * f;
  consumer_sync();
  if (tid < 64) {
    float o[kPConsumerWarps], L[kPConsumerWarps];
#pragma unroll
    for (int v = 0; v < kPConsumerWarps; ++v) {
      o[v] = wacc[v * 64 + tid];
      L[v] = wl[v];
    }
#pragma unroll
    for (int st = kPConsumerWarps / 2; st > 0; st >>= 1)
#pragma unroll
      for (int v = 0; v < st; ++v) {
        o[v] += o[v + st];
        L[v] += L[v + st];
      }
    st_tag(A.attn + h * LE_HEAD_DIM + tid, o[0] / L[0], phase_tag(s, A.layers, l, TG_ATTN));
  }
  if (fine) trace_mark<kTrace>(A, ntr, tok, ftag | 0xC0000u);
  consumer_sync();
}

// Embedding row `token` of the tied lm_head, read from its records, as 8 values per thread
// (elements 8*tid .. 8*tid+7 of the 2048-wide row; dequantize_embedding_row, :182-220).
__device__ __forceinline__ void embed_group(const PArgs& A, int token, float (&v)[8]) {
  const int tid = threadIdx.x & 255;
  const int T = token >> 4, gr = token & 15;
  const uint8_t* rec = A.arena + A.lm_rec_base + (unsigned long long)T * kRecBytes;
  const int b = tid >> 4, q = tid & 15, t = q >> 2, i = q & 3;
  const int L = (gr & 7) * 4 + t, half = gr >> 3;
  const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(rec + b * 1024 + half * 512 + L * 16 + 4 * i));
  const uint32_t sw = __ldg(reinterpret_cast<const uint32_t*>(rec + kRecNibBytes + b * 64 + gr * 4));
  const float st = bf16_bits_to_f32(sw & 0xFFFFu), mv = bf16_bits_to_f32(sw >> 16);
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = __fadd_rn(mv, __fmul_rn((float)((w >> (4 * k)) & 0xFu), st));
}

// ---------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------
// kTrace = true builds the variant that records the phase trace (llama_engine_trace); the
// production variant carries no trace code.
template <bool kTrace>
__global__ void __launch_bounds__(kPThreads, 1) k_decode_persistent(const __grid_constant__ PArgs A) {
  extern __shared__ __align__(1024) uint8_t psmem[];
  uint8_t* ring = psmem;                                          // kRingSlots * kRecBytes
  uint8_t* image = ring + (size_t)kRingSlots * kRecBytes;          // kImageBytes
  float* misc = reinterpret_cast<float*>(image + kImageBytes);     // kMiscFloats
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(misc + kMiscFloats);  // kRingSlots
  uint32_t* s_recs = reinterpret_cast<uint32_t*>(bars + kRingSlots);                     // kMaxRecs
  PItem* s_items = reinterpret_cast<PItem*>(s_recs + kMaxRecs);                          // kMaxItems
  PSeg* s_segs = reinterpret_cast<PSeg*>(s_items + kMaxItems);                           // kMaxSegs
  __shared__ unsigned long long s_best[kPConsumerWarps];
  __shared__ int s_slot_cnt[kRingSlots];  // units done with the record in each slot
  __shared__ int s_token;
  // record index currently issued into each ring slot.  A consumer of record q first waits until
  // its slot holds q: only then does the slot's mbarrier parity refer unambiguously to q (a
  // consumer that ran two uses ahead would otherwise see an older phase of the same parity).
  __shared__ volatile int s_slot_rec[kRingSlots];
  __shared__ volatile int s_fail;  // a ring wait of this CTA gave up: no more copies are issued

  const PCtaSched cs = A.sched[blockIdx.x];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t step_seq = A.ctrl->step_seq, lm_seq = A.ctrl->lm_seq;
  const uint32_t per_tok = A.do_logits ? cs.nrec : cs.nrec_nolm;
  const uint32_t total = per_tok * (uint32_t)A.n_tokens;

  // record q of this launch -> (slot q % kRingSlots, its use count q / kRingSlots)
  auto issue = [&](uint32_t q) {
    const uint32_t slot = q % kRingSlots;
    const unsigned long long off = (unsigned long long)s_recs[q % per_tok] * kRecBytes;
    s_slot_rec[slot] = (int)q;
    mbar_expect_tx(full0 + 8 * slot, kRecBytes);
    bulk_g2s(smem_u32(ring + (size_t)slot * kRecBytes), A.arena + off, kRecBytes, full0 + 8 * slot);
  };

  for (uint32_t i = tid; i < cs.nrec; i += kPThreads) s_recs[i] = A.recs[cs.rec_off + i];
  for (uint32_t i = tid; i < cs.nitem; i += kPThreads) s_items[i] = A.items[cs.item_off + i];
  for (uint32_t i = tid; i < cs.nseg; i += kPThreads) s_segs[i] = A.segs[cs.seg_off + i];
  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < kRingSlots; ++s) {
      mbar_init(full0 + 8 * s, 1);
      s_slot_rec[s] = -1;
      s_slot_cnt[s] = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0)
    for (uint32_t q = 0; q < total && q < (uint32_t)kRingSlots; ++q) issue(q);
  // test only: a wait that no one will satisfy runs out (the error path of every wait)
  if (A.expire_where != 0 && blockIdx.x == 0 && tid == 0)
    wait_counter(A, &A.ctrl->never, 1u, (uint32_t)A.expire_where);

  const int cw = warp;
  Stage S;
  S.bfrag = reinterpret_cast<uint2*>(image);
  S.bsum = reinterpret_cast<float*>(image + 32768);
  S.escl = S.bsum + 64;
  S.red = S.escl + 64;
  int token = A.token0;
  const int pos0 = A.pos0;
  const int L = A.layers;
  int ntr = 0;

  for (int tok = 0; tok < A.n_tokens; ++tok) {
    const uint32_t s = step_seq + (uint32_t)tok;
    const int pos = pos0 + tok;
    const uint32_t rec_base = per_tok * (uint32_t)tok;
    if (tid == 0) trace_mark<kTrace>(A, ntr, tok, 0xFFFF0000u);
    if (tok > 0) {
      // next token = greedy id of the previous step (all CTAs' lm_head work done)
      if (tid == 0) {
        wait_counter(A, &A.ctrl->lm_ctr, (lm_seq + (uint32_t)tok) * (uint32_t)A.n_lm_ctas, 3);
        const unsigned long long k = atomicAdd(&A.ctrl->key[(lm_seq + tok - 1) % 3], 0ull);
        const int t = k == 0ull ? 0 : (int)(~(uint32_t)(k & 0xFFFFFFFFull));
        s_token = (unsigned)t < (unsigned)A.vocab ? t : 0;  // (a failed step leaves no valid key)
      }
      consumer_sync();
      token = s_token;
    }
    // CTA 0 publishes the embedding row as the layer-0 residual x (every CTA dequantises it
    // again for its layer-0 QKV staging, so no register holds it across the segment loop)
    if (blockIdx.x == 0 && tid < 256) {
      float emb[8];
      embed_group(A, token, emb);
      const uint32_t tx = phase_tag(s, L, 0, TG_XIN);
#pragma unroll
      for (int k = 0; k < 8; ++k) st_tag(A.x + 8 * tid + k, emb[k], tx);
      if (tid == 0) {
        A.ctrl->key[(lm_seq + tok + 1) % 3] = 0ull;
        if (tok > 0) A.token_log[tok - 1] = token;
      }
    }

    for (uint32_t si = 0; si < cs.nseg; ++si) {
      const PSeg sg = s_segs[si];
      const int l = sg.layer;
      if (sg.kind == PK_LMHEAD && !A.do_logits) continue;
      const uint32_t tag = ((uint32_t)sg.kind << 8) | (uint32_t)l;
      if (tid == 0) trace_mark<kTrace>(A, ntr, tok, tag | 0x10000u);
      consumer_sync();  // previous segment's readers of the image are done
      if (tid == 0) trace_mark<kTrace>(A, ntr, tok, tag | 0x20000u);
      // o-proj / down: the residual rows were final before this phase; fetch their words now and
      // check the tags in the epilogue
      unsigned long long resw = 0ull;
      if ((sg.kind == PK_O || sg.kind == PK_DOWN) && tid < 16 * (int)(sg.item_end - sg.item_begin))
        resw = ld_tag(A.x + (int)s_items[sg.item_begin + (tid >> 4)].tile * 16 + (tid & 15));
      // ---- staging (the tagged loads are the dependency waits) ----
      switch (sg.kind) {
        case PK_QKV:
          if (l == 0) {
            float emb[8];
            embed_group(A, token, emb);
            float4 gm[2];
            load_gamma(A.norms, gm);
            stage_norm2048_vals(emb, gm, S);
          }
          else stage_norm2048(A, A.x, phase_tag(s, L, l, TG_XIN), A.norms + (size_t)(2 * l) * 2048, S, 10 + l);
          break;
        case PK_ATTN:
          break;
        case PK_O:
          stage_plain(A, A.attn, A.dim, phase_tag(s, L, l, TG_ATTN), S, 200 + l);
          break;
        case PK_GATEUP:
          stage_norm2048(A, A.x, phase_tag(s, L, l, TG_XO), A.norms + (size_t)(2 * l + 1) * 2048, S, 300 + l);
          break;
        case PK_DOWN:
          stage_plain(A, A.act, A.ffn, phase_tag(s, L, l, TG_ACT), S, 400 + l);
          break;
        case PK_LMHEAD:
          stage_norm2048(A, A.x, phase_tag(s, L, L, TG_XIN), A.norms + (size_t)(2 * L) * 2048, S, 500);
          break;
      }
      if (tid == 0) trace_mark<kTrace>(A, ntr, tok, tag | 0x30000u);
      // ---- work ----
      if (sg.kind == PK_ATTN) {
        for (uint32_t it = sg.item_begin; it < sg.item_end; ++it)
          attention_head<kTrace>(A, l, (int)s_items[it].tile, pos, s, misc, reinterpret_cast<float*>(image), ntr, tok);
        if (tid == 0) trace_mark<kTrace>(A, ntr, tok, tag | 0x40000u);
        continue;
      }
      // Work units: the segment's records (consecutive in the CTA's stream, items in order, nrec
      // per item) each split into sg.split block ranges; unit u = (record u / split, range
      // u % split) runs on warp u % 16.  No barrier per record: each unit leaves its 16 row
      // partials in shared memory, and the last unit to finish a ring slot refills it.
      const int SP = sg.split;
      const int n_items = (int)(sg.item_end - sg.item_begin);
      const PItem it0 = s_items[sg.item_begin];
      const int nrec_item = it0.nrec;
      const int n_units = n_items * nrec_item * SP;
      const uint32_t q0 = rec_base + it0.rec;
      float* s_unit = misc;  // [n_units][16]
      // output tags of this phase
      const uint32_t t_out = sg.kind == PK_QKV      ? phase_tag(s, L, l, TG_QKV)
                             : sg.kind == PK_O      ? phase_tag(s, L, l, TG_XO)
                             : sg.kind == PK_GATEUP ? phase_tag(s, L, l, TG_ACT)
                                                    : phase_tag(s, L, l + 1, TG_XIN);
      const uint32_t t_res = sg.kind == PK_O ? phase_tag(s, L, l, TG_XIN) : phase_tag(s, L, l, TG_XO);
      unsigned long long wait_cycles = 0;
      const bool fine = kTrace && tid == 0 && (l == 1 || l == 2);
      for (int u = cw; u < n_units; u += kPConsumerWarps) {
        const int rl = u / SP, sub = u - rl * SP;
        const uint32_t q = q0 + (uint32_t)rl;
        const uint32_t slot = q % kRingSlots;
        const long long w0 = kTrace ? clock64() : 0;
        // after a failed wait (error set) the unit still runs, on whatever the slot holds, and this
        // CTA issues no further copies
        const bool landed = wait_slot(A, s_slot_rec, slot, q, 650 + sg.kind) &&
                            wait_mbar(A, full0 + 8 * slot, (q / kRingSlots) & 1, 600 + sg.kind);
        if (!landed) {
          s_fail = 1;
          __threadfence_block();  // seen by the record's last releaser, after its counter add
        }
        if (kTrace) wait_cycles += (unsigned long long)(clock64() - w0);
        if (fine) trace_mark<kTrace>(A, ntr, tok, tag | 0x70000u);
        float p0, p1;
        record_blocks(SP, ring + (size_t)slot * kRecBytes, sg.kind == PK_DOWN ? rl % nrec_item : 0, sub, S, p0, p1);
        if ((lane & 3) == 0) {
          s_unit[u * 16 + (lane >> 2)] = p0;
          s_unit[u * 16 + (lane >> 2) + 8] = p1;
        }
        if (fine) trace_mark<kTrace>(A, ntr, tok, tag | 0x80000u);
        __syncwarp();  // every lane's reads of the slot have completed
        if (lane == 0) {
          bool last = true;
          if (SP > 1) {
            last = atomicAdd(&s_slot_cnt[slot], 1) == SP - 1;
            if (last) atomicExch(&s_slot_cnt[slot], 0);  // atomic: ordered with the next record's adds
          }
          // only while every wait of this CTA has succeeded: then record q has landed and been
          // read, so the slot holds at most one copy in flight
          if (last && q + kRingSlots < total && !s_fail) issue(q + kRingSlots);
        }
        if (fine) trace_mark<kTrace>(A, ntr, tok, tag | 0x90000u);
      }
      consumer_sync();  // all units' partials are in s_unit
      // epilogue: one thread per (item, row); the residual word was fetched before staging
      unsigned long long best = 0ull;
      for (int e = tid; e < n_items * 16; e += kPThreads) {
        const int i = e >> 4, r = e & 15;
        const int row = (int)s_items[sg.item_begin + i].tile * 16 + r;
        const float* pu = s_unit + (size_t)i * nrec_item * SP * 16 + r;
        if (sg.kind == PK_GATEUP) {  // records: gate, up
          float g = 0.f, up = 0.f;
          for (int v = 0; v < SP; ++v) {
            g += pu[v * 16];
            up += pu[(SP + v) * 16];
          }
          st_tag(A.act + row, (g / (1.0f + expf(-g))) * up, t_out);
          continue;
        }
        float a = 0.f;
        const int nv = nrec_item * SP;
        if (nv == 16) {
          float t[16];
#pragma unroll
          for (int v = 0; v < 16; ++v) t[v] = pu[v * 16];
#pragma unroll
          for (int w = 8; w > 0; w >>= 1)
#pragma unroll
            for (int v = 0; v < w; ++v) t[v] += t[v + w];
          a = t[0];
        } else {
          for (int v = 0; v < nv; ++v) a += pu[v * 16];
        }
        switch (sg.kind) {
          case PK_QKV:
            st_tag(A.qkv + row, a, t_out);
            break;
          case PK_O:
          case PK_DOWN: {
            const float res = (e == tid && tag_of(resw) == t_res) ? tag_val(resw) : ld_tagged1(A, A.x + row, t_res, 700 + l);
            st_tag(A.x + row, res + a, t_out);
            break;
          }
          case PK_LMHEAD:
            A.logits[row] = a;
            if (a > -1e30f) best = max(best, argmax_key(a, row));
            break;
        }
      }
      if (sg.kind == PK_LMHEAD) {
        __threadfence();
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (lane == 0) s_best[cw] = best;
        consumer_sync();
        if (tid == 0) {
          for (int w = 0; w < kPConsumerWarps; ++w) best = max(best, s_best[w]);
          atomicMax(&A.ctrl->key[(lm_seq + tok) % 3], best);
          __threadfence();
          atomicAdd(&A.ctrl->lm_ctr, 1u);
        }
      }
      if (cw == 0 && lane == 0) trace_mark<kTrace>(A, ntr, tok, tag | 0x50000u, wait_cycles | 1ull);
      if (tid == 0) trace_mark<kTrace>(A, ntr, tok, tag | 0x40000u);
    }
  }

  // ---------------- launch epilogue ----------------
  __syncthreads();
  if (tid == 0) {
    // every issued copy has been consumed, unless a wait gave up: make sure none is in flight
    // (the last copy issued into each slot has landed; earlier ones were waited for before it)
    for (int sl = 0; sl < kRingSlots; ++sl) {
      const int qlast = s_slot_rec[sl];
      if (qlast >= 0) wait_mbar_drain(A, full0 + 8 * sl, ((uint32_t)qlast / kRingSlots) & 1, 2);
    }
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
      if (A.host_done) {
        volatile uint32_t* hd = A.host_done;
        hd[0] = *reinterpret_cast<volatile uint32_t*>(&A.ctrl->error);
        hd[1] = *reinterpret_cast<volatile uint32_t*>(&A.ctrl->err_where);
        hd[2] = (uint32_t)*reinterpret_cast<volatile int32_t*>(A.am_result);
        __threadfence_system();
        hd[3] = A.seq;
      }
    }
  }
}

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
      *reinterpret_cast<uint4*>(rec + j * 1024 + half * 512 + L * 16) = v;
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
