// Engine state and the llama_engine.h C ABI for the B200 (sm_100a) build.
//
// Host side of the drop-in: parses and validates the LLM4S128 file (the reference does the same
// parse without validation, src/llama_engine.cpp:865-906), uploads every array into one device
// arena, builds the RoPE table on the host with the reference's own libm calls (:908-917) so
// the table is bit-identical, allocates device KV caches, and captures the per-token kernel
// sequence into CUDA graphs.
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "batch_kernels.cuh"
#include "decode_kernels.cuh"
#include "mma_gemv.cuh"
#include "persistent.cuh"
#include "tc_gemm.cuh"
#include "attn_tc.cuh"
#include "llama_engine.h"
#include <nccl.h>

#define LE_API extern "C" __attribute__((visibility("default")))

namespace le {

static std::mutex g_err_mu;
static std::string g_create_error = "";

static void set_create_error(const std::string& s) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  g_create_error = s;
}

// Restores the caller's current CUDA device on scope exit.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

struct FileMatrix {
  uint32_t N = 0, K = 0, nb = 0;
  size_t nib_off = 0, step_off = 0, min_off = 0;  // byte offsets into the file
};

struct FileLayer {
  size_t in_norm_off = 0, post_norm_off = 0;
  FileMatrix m[7];  // q k v o gate up down
};

struct ParsedFile {
  uint32_t layers, dim, ffn, vocab, heads, kv_heads, block;
  size_t final_norm_off;
  std::vector<FileLayer> L;
  FileMatrix lm_head;
};

// Parses the header and walks the matrix records, checking every size against the file length.
static bool parse_file(const uint8_t* base, size_t size, ParsedFile& P, std::string& err) {
  if (size < 36) { err = "file shorter than the LLM4S128 header"; return false; }
  if (std::memcmp(base, "LLM4S128", 8) != 0) { err = "bad magic (expected LLM4S128)"; return false; }
  uint32_t h[7];
  std::memcpy(h, base + 8, 28);
  P.layers = h[0]; P.dim = h[1]; P.ffn = h[2]; P.vocab = h[3]; P.heads = h[4]; P.kv_heads = h[5]; P.block = h[6];
  if (P.block != 128) { err = "block size must be 128"; return false; }
  if (P.layers == 0 || P.dim == 0 || P.ffn == 0 || P.vocab == 0 || P.heads == 0 || P.kv_heads == 0 ||
      P.dim % P.heads != 0 || P.heads % P.kv_heads != 0) {
    err = "inconsistent model dimensions"; return false;
  }
  if (P.dim / P.heads != LE_HEAD_DIM) { err = "head_dim must be 64"; return false; }
  if (P.dim % 1024 != 0 || P.ffn % 1024 != 0) { err = "dim and ffn_dim must be multiples of 1024"; return false; }
  if (P.dim > 16384 || P.ffn > 65536 || P.layers > 1024) { err = "model dimensions out of supported range"; return false; }
  size_t off = 36;
  auto need = [&](size_t n) { return off + n <= size; };
  auto take_norm = [&](size_t& where) -> bool {
    if (!need((size_t)P.dim * 4)) return false;
    where = off; off += (size_t)P.dim * 4; return true;
  };
  auto take_mat = [&](FileMatrix& m, uint32_t N, uint32_t K) -> bool {
    if (!need(12)) return false;
    uint32_t hh[3];
    std::memcpy(hh, base + off, 12);
    off += 12;
    if (hh[0] != N || hh[1] != K || (uint64_t)hh[2] != (uint64_t)N * (K / 128)) return false;
    m.N = N; m.K = K; m.nb = hh[2];
    if (!need((size_t)m.nb * 68)) return false;
    m.nib_off = off; off += (size_t)m.nb * 64;
    m.step_off = off; off += (size_t)m.nb * 2;
    m.min_off = off; off += (size_t)m.nb * 2;
    return true;
  };
  if (!take_norm(P.final_norm_off)) { err = "file truncated (final_norm)"; return false; }
  const uint32_t kvd = P.kv_heads * LE_HEAD_DIM;
  const uint32_t shapes[7][2] = {{P.dim, P.dim}, {kvd, P.dim}, {kvd, P.dim}, {P.dim, P.dim},
                                 {P.ffn, P.dim}, {P.ffn, P.dim}, {P.dim, P.ffn}};
  P.L.resize(P.layers);
  for (uint32_t l = 0; l < P.layers; ++l) {
    if (!take_norm(P.L[l].in_norm_off) || !take_norm(P.L[l].post_norm_off)) {
      err = "file truncated (layer norms)"; return false;
    }
    for (int i = 0; i < 7; ++i)
      if (!take_mat(P.L[l].m[i], shapes[i][0], shapes[i][1])) {
        err = "matrix record " + std::to_string(i) + " of layer " + std::to_string(l) +
              " is truncated or has an unexpected shape";
        return false;
      }
  }
  if (!take_mat(P.lm_head, P.vocab, P.dim)) { err = "lm_head record truncated or mis-shaped"; return false; }
  return true;
}

struct DevLayer {
  const float* in_norm;
  const float* post_norm;
  QMat q, k, v, o, g, u, d;
};

constexpr int kRing = 64;

// Weight records of one tensor-core GEMM (row tiles x K blocks, tc_gemm.cuh layout).
struct TcMat {
  const uint8_t* recs = nullptr;
  int tiles = 0, kb = 0;
};
struct TcLayer {
  TcMat qkv, o, gu, d;
};
constexpr int kTcMaxSplits = 8;
// Two-tile GEMM units where they are estimated faster (tc_plan), on unless $LLAMA_B200_TC_PAIR is
// "0" (read once).
static bool tc_pair_enabled() {
  static const bool on = [] {
    const char* v = getenv("LLAMA_B200_TC_PAIR");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}
constexpr int kExpireAttn = 20;  // llama_engine_debug_waits code that expires only the prefill attention
constexpr int kAttnMaxSplits = 8;
constexpr int kScoreRows = 256;  // rows of logits held at once by llama_engine_score_tokens

struct Engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t layers = 0, dim = 0, ffn = 0, vocab = 0, heads = 0, kv_heads = 0, kv_dim = 0;
  int max_batch = 1, max_seq = LE_MAX_SEQ_LEN;
  int num_sms = 148;

  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  const float* final_norm = nullptr;
  std::vector<DevLayer> L;
  QMat lm_head{};

  float* rope_cos = nullptr;  // [LE_MAX_SEQ_LEN][32], bit-identical to the reference table
  float* rope_sin = nullptr;
  float* kcache = nullptr;    // [slot][layer][max_seq][kv_dim]
  float* vcache = nullptr;

  // activations
  float* x = nullptr;      // [max_batch][dim]   residual stream
  float* qkv = nullptr;    // [max_batch][dim + 2 kv_dim]
  float* attn = nullptr;   // [max_batch][dim]
  float* act = nullptr;    // [max_batch][ffn]
  float* logits = nullptr; // [max_batch][vocab]
  float* emb = nullptr;    // [dim] scratch for llama_engine_dequantize_embedding
  float* red = nullptr;    // [2048] partial reductions of the sampler
  int32_t* d_misc = nullptr;  // [16] small device scalars (embedding row id)
  ArgmaxPart* part = nullptr;  // [max_batch][lm_grid]
  int32_t* am_result = nullptr;  // [max_batch]
  int32_t* token_log = nullptr;  // [LE_MAX_SEQ_LEN]
  StepParams* d_params = nullptr;  // [max_batch]
  int lm_grid = 0;

  // host side
  StepParams* h_ring = nullptr;  // pinned
  cudaEvent_t ring_ev[kRing] = {};
  bool ring_used[kRing] = {};
  int ring_pos = 0;
  int32_t last_pos = 0;  // last position queued for slot 0 (diagnostics re-use it)
  float* h_logits = nullptr;  // pinned [max_batch][vocab]
  int32_t* h_small = nullptr; // pinned scratch [LE_MAX_SEQ_LEN]
  bool logits_on_host_fresh = false;   // slot-0 host mirror matches device
  bool argmax_valid = false;           // am_result[0] holds greedy of current device logits
  bool argmax_persist = false;         // ... from the newest persistent launch (also in h_done)
  uint32_t* h_done = nullptr;          // mapped pinned words the persistent kernel's last CTA writes
  uint32_t persist_seq = 0;            // persistent launches so far
  uint32_t persist_seq_logits = 0;     // the newest one with logits
  bool have_logits = false;

  // persistent token-step kernel (LLaMA-3.2-1B geometry: dim 2048, ffn 8192)
  bool persist = false;
  uint8_t* rec_arena = nullptr;
  size_t rec_bytes = 0;
  PCtaSched* d_sched = nullptr;
  PSeg* d_segs = nullptr;
  PItem* d_items = nullptr;
  uint32_t* d_recs = nullptr;
  float* d_norms = nullptr;  // [2*layers + 1][dim] contiguous copy of the norm weights
  unsigned long long* d_tagged = nullptr;  // x | qkv | attn | act as (value, phase tag) words
  uint8_t* ctrl_block = nullptr;  // PCtrl, then am_result [max_batch]
  PCtrl* d_ctrl = nullptr;        // the start of ctrl_block (persistent kernel only)
  uint32_t* h_err = nullptr;  // pinned mirror of PCtrl::error / err_where
  unsigned long long* d_trace = nullptr;  // optional phase trace of the persistent kernel
  PArgs pargs{};
  int p_grid = 0;

  // token-batched path: tensor-core GEMMs over tc_T tokens at most per step
  bool tc = false;
  int tc_T = 0;
  uint8_t* tc_arena = nullptr;
  std::vector<TcLayer> tcl;
  TcMat tc_lm;
  uint8_t* img_d = nullptr;  // activation images, K = dim   [tc_T/64][dim/128][kImgBytes]
  uint8_t* img_f = nullptr;  //                      K = ffn
  float* t_x = nullptr;      // [tc_T][dim] residual stream
  float* t_q = nullptr;      // [tc_T][dim] rotated queries
  float* t_attn = nullptr;   // [tc_T][dim]
  float* t_qkv = nullptr;    // [kTcMaxSplits][tc_T][dim + 2 kv_dim] q | k | v before RoPE (split-K planes)
  float* t_gu = nullptr;     // [tc_T][ffn] SiLU(gate) * up, from the gate-up GEMM's epilogue
  float* t_part = nullptr;   // [kTcMaxSplits][tc_T][dim] split-K partial sums
  float* t_attn_part = nullptr;  // [tc_T][kv_heads][kAttnMaxSplits][kAttnPart] attention partials
  uint8_t* kv_img = nullptr;     // [kv_heads][kv_img_tiles] prefill K / V tile images (attn::kTileBytes)
  int kv_img_tiles = 0;          // tiles per kv head: ceil(max_seq / 64)
  int32_t* t_idx = nullptr;  // [3][tc_T] token | position | slot of the step's rows
  int32_t* h_idx = nullptr;  // pinned staging of t_idx
  cudaEvent_t idx_ev = nullptr;
  bool idx_pending = false;
  ArgmaxPart* t_am = nullptr;  // [tc_T][tc_am_parts]
  int tc_am_parts = 0;
  uint32_t* tc_err = nullptr;  // device error word of the tensor-core GEMM
  bool tc_dirty = true;        // a batched step ran since tc_err was last read
  unsigned long long tc_wait_ns = kWaitNs;  // bound on the GEMM's waits (test hook)
  int tc_expire = 0;                        // test hook: the GEMM's issuer waits on nothing
  int attn_expire = 0;                      // test hook: the prefill attention's issuer waits on nothing
  unsigned long long attn_wait_ns = kWaitNs;  // bound on the prefill attention's waits (test hook)
  // decode steps of the batched path replayed as CUDA graphs, one per (rows, logits rows,
  // attention splits); the rows' ids, positions and slots are read from t_idx
  struct TcGraph { int n, nlog, splits; bool fold; cudaGraphExec_t exec; };
  std::vector<TcGraph> tc_graphs;
  // token scoring (llama_engine_score_tokens): logits of a chunk's rows, targets, results
  float* sc_logits = nullptr;   // [kScoreRows][vocab], allocated on first use
  int32_t* sc_target = nullptr; // [kScoreRows]
  float* sc_lp = nullptr;       // [kScoreRows]
  int32_t* sc_greedy = nullptr; // [kScoreRows]

  cudaGraphExec_t g_fwd[2] = {nullptr, nullptr};  // [compute_logits]
  cudaGraphExec_t g_gen = nullptr;                // forward + greedy + advance

  // 2-way tensor-parallel batch-1 variant (tp_world == 2): this rank's share of every layer
  int tp_world = 1, tp_rank = 0;
  ncclComm_t tp_comm = nullptr;
  uint8_t* tp_arena = nullptr;      // column halves of W_o and W_down
  std::vector<DevLayer> tpl;        // row slices (q, k, v, gate, up) and column halves (o, down)
  QMat tp_lm{};                     // this rank's vocabulary rows of the lm_head
  float* tp_kc = nullptr;           // [layers][max_seq][kv_dim / 2]
  float* tp_vc = nullptr;
  float* tp_qkv = nullptr;          // [(dim + 2 kv_dim) / 2]
  float* tp_attn = nullptr;         // [dim / 2]
  float* tp_act = nullptr;          // [ffn / 2]
  ArgmaxPart* tp_part = nullptr;    // [lm_grid]
  int32_t* tp_cand = nullptr;       // [world][2]: (value bits, global index) of each rank's greedy candidate
  cudaGraphExec_t tp_g[3] = {nullptr, nullptr, nullptr};  // no logits | logits (gathered) | greedy + advance

  std::string err;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

#define LE_CK(expr)                                                          \
  do {                                                                       \
    cudaError_t e_ = (expr);                                                 \
    if (e_ != cudaSuccess) {                                                 \
      E->err = std::string(#expr) + ": " + cudaGetErrorString(e_);           \
      return false;                                                          \
    }                                                                        \
  } while (0)

// ---------------------------------------------------------------------------------------------
// Kernel sequence of one token for one sequence.
// ---------------------------------------------------------------------------------------------
static size_t gemv_smem(int K, int mx = 1) { return (size_t)mx * (K + K / 128) * 4 + 32 * 4 + 64; }

static bool set_smem_attrs(Engine* E) {
  LE_CK(cudaFuncSetAttribute(k_proj_residual<1, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)gemv_smem(E->ffn)));
  return true;
}

struct TokenBuffers {
  const StepParams* prm;  // device params for this row
  float* x;
  float* qkv;
  float* attn;
  float* act;
  float* kc;  // KV base of the slot (layer 0)
  float* vc;
  float* logits;  // nullptr: no lm_head
  ArgmaxPart* part;
  int32_t* result;
  StepParams* prm_mut;  // for advance
  int32_t* token_log;
  int advance;
};

enum Phase { PH_QKV = 0, PH_ATTN, PH_OPROJ, PH_GATEUP, PH_DOWN, PH_LMHEAD };

// Enqueues one phase of the token step for layer l (PH_LMHEAD ignores l).
static void enqueue_phase(Engine* E, const TokenBuffers& B, int phase, uint32_t l, cudaStream_t s) {
  const int dim = E->dim, ffn = E->ffn, kvd = E->kv_dim;
  const size_t layer_stride = (size_t)E->max_seq * kvd;
  const DevLayer& Ly = E->L[l];
  switch (phase) {
    case PH_QKV: {
      const int grid = ((dim + 2 * kvd) / 2 + kWarps - 1) / kWarps;
      k_qkv<2><<<grid, kThreads, gemv_smem(dim), s>>>(B.x, Ly.in_norm, Ly.q, Ly.k, Ly.v, B.qkv);
      break;
    }
    case PH_ATTN: {
      const size_t att_smem = (size_t)(64 * 3 + 32 + 256 + E->max_seq) * 4;
      k_attention<<<E->heads, kThreads, att_smem, s>>>(B.qkv, B.kc + l * layer_stride, B.vc + l * layer_stride,
                                                        E->rope_cos, E->rope_sin, B.prm, E->heads, E->kv_heads,
                                                        B.attn);
      break;
    }
    case PH_OPROJ:
      k_proj_residual<1, 2><<<(dim + kWarps - 1) / kWarps, kThreads, gemv_smem(dim), s>>>(B.attn, Ly.o, B.x);
      break;
    case PH_GATEUP:
      k_gateup<2><<<(ffn / 2 + kWarps - 1) / kWarps, kThreads, gemv_smem(dim), s>>>(B.x, Ly.post_norm, Ly.g, Ly.u,
                                                                                   B.act);
      break;
    case PH_DOWN:
      k_proj_residual<1, 8><<<(dim + kWarps - 1) / kWarps, kThreads, gemv_smem(ffn), s>>>(B.act, Ly.d, B.x);
      break;
    case PH_LMHEAD:
      k_lmhead<2><<<E->lm_grid, kThreads, gemv_smem(dim), s>>>(B.x, E->final_norm, E->lm_head,
                                                               B.logits ? B.logits : E->logits, B.part);
      break;
  }
}

static void enqueue_token(Engine* E, const TokenBuffers& B, cudaStream_t s) {
  k_embed<<<1, kThreads, 0, s>>>(E->lm_head, B.prm, nullptr, B.x);
  for (uint32_t l = 0; l < E->layers; ++l)
    for (int ph = PH_QKV; ph <= PH_DOWN; ++ph) enqueue_phase(E, B, ph, l, s);
  if (B.logits) {
    enqueue_phase(E, B, PH_LMHEAD, 0, s);
    k_argmax_finish<<<1, 1024, 0, s>>>(B.part, E->lm_grid, B.result, B.prm_mut, B.token_log, B.advance);
  }
}

static TokenBuffers row_buffers(Engine* E, int row, int slot, bool logits, int advance) {
  TokenBuffers B;
  B.prm = E->d_params + row;
  B.prm_mut = E->d_params + row;
  B.x = E->x + (size_t)row * E->dim;
  B.qkv = E->qkv + (size_t)row * (E->dim + 2 * E->kv_dim);
  B.attn = E->attn + (size_t)row * E->dim;
  B.act = E->act + (size_t)row * E->ffn;
  const size_t slot_stride = (size_t)E->layers * E->max_seq * E->kv_dim;
  B.kc = E->kcache + (size_t)slot * slot_stride;
  B.vc = E->vcache + (size_t)slot * slot_stride;
  B.logits = logits ? E->logits + (size_t)row * E->vocab : nullptr;
  B.part = E->part + (size_t)row * E->lm_grid;
  B.result = E->am_result + row;
  B.token_log = E->token_log;
  B.advance = advance;
  return B;
}

static bool capture(Engine* E, const TokenBuffers& B, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  LE_CK(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  enqueue_token(E, B, E->stream);
  cudaError_t ce = cudaStreamEndCapture(E->stream, &g);
  if (ce != cudaSuccess) { E->err = std::string("capture: ") + cudaGetErrorString(ce); return false; }
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) { E->err = std::string("instantiate: ") + cudaGetErrorString(ce); return false; }
  return true;
}

static void destroy(Engine* E);

// ---------------------------------------------------------------------------------------------
// Persistent kernel set-up: record arena, static schedule, control words.
// ---------------------------------------------------------------------------------------------
static bool persistent_supported(const Engine* E) {
  const char* v = getenv("LLAMA_B200_PERSISTENT");
  if (v && std::strcmp(v, "0") == 0) return false;
  return E->dim == 2048 && (E->ffn == 2048 || E->ffn == 4096 || E->ffn == 8192) && E->vocab % 16 == 0 &&
         E->kv_dim % 16 == 0 &&
         (E->dim + 2 * E->kv_dim) % 16 == 0;
}

static size_t persistent_smem() {
  return (size_t)kRingSlots * kRecBytes + kImageBytes + kMiscFloats * 4 + kRingSlots * 8 + kSchedBytes;
}

// ---------------------------------------------------------------------------------------------
// Static schedule of the persistent kernel (host only, no device calls).
// ---------------------------------------------------------------------------------------------
struct PGeom { int layers, dim, ffn, vocab, heads, kv_heads; };

struct PSchedule {
  // record arena: per layer [q|k|v tiles][o tiles][gate tiles][up tiles][down tiles x ffn/2048],
  // then the lm_head tiles
  size_t rec_qkv = 0, rec_o = 0, rec_g = 0, rec_d = 0, rec_lm = 0, per_layer = 0, lm_base = 0, nrec_total = 0;
  size_t layer_base(int l) const { return (size_t)l * per_layer; }
  std::vector<PCtaSched> sched;
  std::vector<PSeg> segs;
  std::vector<PItem> items;
  std::vector<uint32_t> recs;
  int n_lm_ctas = 0;
};

// Every phase hands out whole items (16-row tiles with their records) round-robin over the CTAs,
// continuing where the previous phase stopped; attention heads are spread over the grid.  Inside
// a CTA a segment's records are cut into work units of 16 / split blocks (split chosen per
// segment by choose_split).
static bool build_schedule(const PGeom& g, int G, PSchedule& P, std::string& err) {
  const int L = g.layers, kv_dim = g.kv_heads * LE_HEAD_DIM;
  P.rec_qkv = (size_t)(g.dim + 2 * kv_dim) / 16;
  P.rec_o = (size_t)g.dim / 16;
  P.rec_g = (size_t)g.ffn / 16;
  P.rec_d = (size_t)(g.dim / 16) * (g.ffn / 2048);
  P.rec_lm = (size_t)g.vocab / 16;
  P.per_layer = P.rec_qkv + P.rec_o + 2 * P.rec_g + P.rec_d;
  P.lm_base = P.per_layer * L;
  P.nrec_total = P.lm_base + P.rec_lm;
  struct CtaLists { std::vector<PSeg> segs; std::vector<PItem> items; std::vector<uint32_t> recs; };
  // Work units per record for a segment of n_rec records: the split (block ranges of 16/split
  // blocks) that minimises the busiest warp's (units x (blocks per unit + 2)), the 2 standing
  // for a unit's fixed cost, within the shared-memory room for unit partials.
  auto choose_split = [](int n_rec) -> int {  // splits 2..16 (a unit covers at most 8 blocks)
    int best = 2, best_cost = 1 << 30;
    for (int sp = 2; sp <= 16; sp *= 2) {
      if (n_rec * sp > kMaxUnits) break;
      const int units_per_warp = (n_rec * sp + kPConsumerWarps - 1) / kPConsumerWarps;
      const int cost = units_per_warp * (16 / sp + 2);
      if (cost < best_cost) { best_cost = cost; best = sp; }
    }
    return best;
  };
  bool fits = true;
  std::vector<CtaLists> C(G);
  int rot = 0;
  auto add_phase = [&](uint16_t kind, int layer, int n_items, int nrec_per_item,
                       const std::function<size_t(int, int)>& rec_of, const std::function<int(int)>& cta_of) {
    std::vector<std::vector<int>> per(G);
    for (int i = 0; i < n_items; ++i) per[cta_of(i)].push_back(i);
    for (int c = 0; c < G; ++c) {
      if (per[c].empty()) continue;
      PSeg sg{};
      sg.kind = (uint8_t)kind;
      sg.layer = (uint16_t)layer;
      sg.item_begin = (uint16_t)C[c].items.size();
      for (int i : per[c]) {
        PItem it{};
        it.kind = (uint8_t)kind;
        it.layer = (uint16_t)layer;
        it.tile = (uint16_t)i;
        it.rec = (uint16_t)C[c].recs.size();
        it.nrec = (uint8_t)nrec_per_item;
        for (int r = 0; r < nrec_per_item; ++r) C[c].recs.push_back((uint32_t)rec_of(i, r));
        C[c].items.push_back(it);
      }
      sg.item_end = (uint16_t)C[c].items.size();
      const int n_rec = (int)per[c].size() * nrec_per_item;
      sg.split = (uint8_t)choose_split(n_rec);
      if (n_rec * sg.split > kMaxUnits) fits = false;
      C[c].segs.push_back(sg);
    }
  };
  const int n_qkv = (int)P.rec_qkv, n_o = (int)P.rec_o, n_gu = (int)P.rec_g, n_down = g.dim / 16;
  const int kq_down = g.ffn / 2048, n_lm = (int)P.rec_lm;
  for (int l = 0; l < L; ++l) {
    const size_t b = P.layer_base(l);
    int r0 = rot;
    add_phase(PK_QKV, l, n_qkv, 1, [&](int i, int) { return b + i; }, [&](int i) { return (r0 + i) % G; });
    rot = (rot + n_qkv) % G;
    add_phase(PK_ATTN, l, g.heads, 0, [&](int, int) { return (size_t)0; },
              [&](int h) { return (int)(((long long)h * G) / g.heads + G / (2 * g.heads)) % G; });
    r0 = rot;
    add_phase(PK_O, l, n_o, 1, [&](int i, int) { return b + P.rec_qkv + i; }, [&](int i) { return (r0 + i) % G; });
    rot = (rot + n_o) % G;
    r0 = rot;
    add_phase(PK_GATEUP, l, n_gu, 2,
              [&](int i, int r) { return b + P.rec_qkv + P.rec_o + (r == 0 ? 0 : P.rec_g) + i; },
              [&](int i) { return (r0 + i) % G; });
    rot = (rot + n_gu) % G;
    r0 = rot;
    add_phase(PK_DOWN, l, n_down, kq_down,
              [&](int i, int r) { return b + P.rec_qkv + P.rec_o + 2 * P.rec_g + (size_t)i * kq_down + r; },
              [&](int i) { return (r0 + i) % G; });
    rot = (rot + n_down) % G;
  }
  std::vector<uint32_t> nrec_nolm(G);
  for (int c = 0; c < G; ++c) nrec_nolm[c] = (uint32_t)C[c].recs.size();
  {
    const int r0 = rot;
    add_phase(PK_LMHEAD, L, n_lm, 1, [&](int i, int) { return P.lm_base + i; }, [&](int i) { return (r0 + i) % G; });
  }
  P.n_lm_ctas = 0;
  for (int c = 0; c < G; ++c)
    for (const auto& sg : C[c].segs)
      if (sg.kind == PK_LMHEAD) ++P.n_lm_ctas;
  for (int c = 0; c < G; ++c)
    if (C[c].recs.size() > (size_t)kMaxRecs || C[c].items.size() > (size_t)kMaxItems ||
        C[c].segs.size() > (size_t)kMaxSegs)
      fits = false;
  if (!fits) { err = "a CTA's schedule exceeds its shared-memory capacity"; return false; }
  P.sched.assign(G, PCtaSched{});
  for (int c = 0; c < G; ++c) {
    PCtaSched& cs = P.sched[c];
    cs.seg_off = (uint32_t)P.segs.size();
    cs.nseg = (uint32_t)C[c].segs.size();
    cs.item_off = (uint32_t)P.items.size();
    cs.nitem = (uint32_t)C[c].items.size();
    cs.rec_off = (uint32_t)P.recs.size();
    cs.nrec = (uint32_t)C[c].recs.size();
    cs.nrec_nolm = nrec_nolm[c];
    P.segs.insert(P.segs.end(), C[c].segs.begin(), C[c].segs.end());
    P.items.insert(P.items.end(), C[c].items.begin(), C[c].items.end());
    P.recs.insert(P.recs.end(), C[c].recs.begin(), C[c].recs.end());
  }
  return true;
}

// Host check of a schedule against the arena layout, reading every entry the way the kernel
// does: every (phase, layer, tile) is one item of exactly one CTA, and its records are that
// tile's records of the right matrices (gate then up; the down row's 2048-column groups in
// order); items and records are consumed in stream order; segments run in phase order; every
// attention head runs once per layer; units fit the shared-memory partials.
static bool check_schedule(const PGeom& g, int G, const PSchedule& P, std::string& err) {
  const int L = g.layers, KQd = g.ffn / 2048;
  struct RecInfo { int kind, layer, tile, sub; };  // sub: gate 0 / up 1, or the down kq
  auto rec_info = [&](size_t r) -> RecInfo {
    if (r >= P.nrec_total) return {-1, -1, -1, -1};
    if (r >= P.lm_base) return {PK_LMHEAD, L, (int)(r - P.lm_base), 0};
    const int l = (int)(r / P.per_layer);
    size_t o = r % P.per_layer;
    if (o < P.rec_qkv) return {PK_QKV, l, (int)o, 0};
    o -= P.rec_qkv;
    if (o < P.rec_o) return {PK_O, l, (int)o, 0};
    o -= P.rec_o;
    if (o < 2 * P.rec_g) return {PK_GATEUP, l, (int)(o % P.rec_g), (int)(o / P.rec_g)};
    o -= 2 * P.rec_g;
    return {PK_DOWN, l, (int)(o / KQd), (int)(o % KQd)};
  };
  auto ntiles_of = [&](int kind) -> int {
    switch (kind) {
      case PK_QKV: return (int)P.rec_qkv;
      case PK_ATTN: return g.heads;
      case PK_O: return (int)P.rec_o;
      case PK_GATEUP: return (int)P.rec_g;
      case PK_DOWN: return g.dim / 16;
      default: return (int)P.rec_lm;
    }
  };
  auto nrec_of = [&](int kind) { return kind == PK_ATTN ? 0 : kind == PK_GATEUP ? 2 : kind == PK_DOWN ? KQd : 1; };
  std::map<std::pair<int, int>, std::vector<int>> seen;  // (kind, layer) -> items per tile
  auto fail = [&](int c, const std::string& m) { err = "schedule check, CTA " + std::to_string(c) + ": " + m; return false; };
  for (int c = 0; c < G; ++c) {
    const PCtaSched& cs = P.sched[c];
    int next_item = 0, next_rec = 0, prev_order = -1;
    for (uint32_t si = 0; si < cs.nseg; ++si) {
      const PSeg& sg = P.segs[cs.seg_off + si];
      const int order = sg.kind == PK_LMHEAD ? 1 << 30 : sg.layer * 8 + sg.kind;
      if (order <= prev_order) return fail(c, "segments out of phase order");
      prev_order = order;
      if (sg.item_begin != next_item || sg.item_end <= sg.item_begin || sg.item_end > cs.nitem)
        return fail(c, "segment items not contiguous");
      if (sg.kind != PK_ATTN && sg.split != 2 && sg.split != 4 && sg.split != 8 && sg.split != 16)
        return fail(c, "bad split");
      int seg_recs = 0;
      auto& cov = seen[{sg.kind, sg.layer}];
      if (cov.empty()) cov.assign(ntiles_of(sg.kind), 0);
      for (int it = sg.item_begin; it < sg.item_end; ++it) {
        const PItem& item = P.items[cs.item_off + it];
        if (item.kind != sg.kind || item.layer != sg.layer) return fail(c, "item of another phase");
        if (item.tile >= cov.size()) return fail(c, "tile out of range");
        cov[item.tile]++;
        if (item.nrec != nrec_of(sg.kind)) return fail(c, "wrong record count");
        if (sg.kind == PK_ATTN) continue;
        if (item.rec != next_rec) return fail(c, "records not in stream order");
        for (int k = 0; k < item.nrec; ++k) {
          const RecInfo ri = rec_info(P.recs[cs.rec_off + item.rec + k]);
          if (ri.kind != sg.kind || ri.layer != (sg.kind == PK_LMHEAD ? L : sg.layer) || ri.tile != item.tile ||
              ri.sub != (sg.kind == PK_GATEUP || sg.kind == PK_DOWN ? k : 0))
            return fail(c, "record does not belong to its item");
        }
        next_rec += item.nrec;
        seg_recs += item.nrec;
      }
      if (sg.kind != PK_ATTN && seg_recs * sg.split > kMaxUnits) return fail(c, "too many units in a segment");
      if (sg.kind != PK_LMHEAD && (uint32_t)next_rec > cs.nrec_nolm) return fail(c, "records before the lm_head");
      next_item = sg.item_end;
    }
    if ((uint32_t)next_item != cs.nitem || (uint32_t)next_rec != cs.nrec) return fail(c, "item/record totals");
  }
  for (int l = 0; l < L; ++l)
    for (int kind : {PK_QKV, PK_ATTN, PK_O, PK_GATEUP, PK_DOWN}) {
      auto it = seen.find({kind, l});
      if (it == seen.end()) { err = "schedule check: a phase has no work"; return false; }
      for (int v : it->second)
        if (v != 1) { err = "schedule check: a tile or head is not handled exactly once"; return false; }
    }
  auto it = seen.find({PK_LMHEAD, L});
  if (it == seen.end()) { err = "schedule check: no lm_head work"; return false; }
  for (int v : it->second)
    if (v != 1) { err = "schedule check: an lm_head tile is not handled exactly once"; return false; }
  return true;
}

static bool init_persistent(Engine* E) {
  if (!persistent_supported(E)) return true;
  const int L = (int)E->layers, G = E->num_sms;
  const size_t smem = persistent_smem();
  LE_CK(cudaFuncSetAttribute(k_decode_persistent<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  LE_CK(cudaFuncSetAttribute(k_decode_persistent<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  LE_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_persistent<false>, kPThreads, smem));
  int per_sm_trace = 0;
  LE_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_trace, k_decode_persistent<true>, kPThreads, smem));
  per_sm = std::min(per_sm, per_sm_trace);
  if (per_sm < 1) {  // keep the kernel-chain path, and say why
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, k_decode_persistent<false>);
    E->err = "persistent kernel declined: 0 resident CTAs per SM (regs " + std::to_string(fa.numRegs) +
             ", static smem " + std::to_string(fa.sharedSizeBytes) + ", dynamic smem " + std::to_string(smem) +
             ", max threads " + std::to_string(fa.maxThreadsPerBlock) + ")";
    return true;
  }
  PGeom geo{L, (int)E->dim, (int)E->ffn, (int)E->vocab, (int)E->heads, (int)E->kv_heads};
  PSchedule P;
  std::string serr;
  if (!build_schedule(geo, G, P, serr) || !check_schedule(geo, G, P, serr)) {
    E->err = "persistent kernel declined: " + serr;
    return true;  // keep the kernel-chain path
  }
  E->rec_bytes = P.nrec_total * kRecBytes;
  LE_CK(cudaMalloc(&E->rec_arena, E->rec_bytes));
  auto repack = [&](const QMat& W, size_t rec0) -> bool {
    k_repack<<<E->num_sms * 8, 256, 0, E->stream>>>(W, E->rec_arena + rec0 * kRecBytes);
    LE_CK(cudaGetLastError());
    return true;
  };
  for (int l = 0; l < L; ++l) {
    const DevLayer& D = E->L[l];
    size_t b = P.layer_base(l);
    if (!repack(D.q, b)) return false;
    if (!repack(D.k, b + E->dim / 16)) return false;
    if (!repack(D.v, b + (E->dim + E->kv_dim) / 16)) return false;
    b += P.rec_qkv;
    if (!repack(D.o, b)) return false;
    b += P.rec_o;
    if (!repack(D.g, b)) return false;
    if (!repack(D.u, b + P.rec_g)) return false;
    b += 2 * P.rec_g;
    if (!repack(D.d, b)) return false;
  }
  if (!repack(E->lm_head, P.lm_base)) return false;
  const std::vector<PCtaSched>& sched = P.sched;
  const std::vector<PSeg>& segs = P.segs;
  const std::vector<PItem>& items = P.items;
  const std::vector<uint32_t>& recs = P.recs;
  const int n_lm_ctas = P.n_lm_ctas;
  const size_t lm_base = P.lm_base;
  auto upload = [&](void** dst, const void* src, size_t bytes) -> bool {
    LE_CK(cudaMalloc(dst, std::max<size_t>(bytes, 16)));
    if (bytes) LE_CK(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
    return true;
  };
  if (!upload((void**)&E->d_sched, sched.data(), sched.size() * sizeof(PCtaSched))) return false;
  if (!upload((void**)&E->d_segs, segs.data(), segs.size() * sizeof(PSeg))) return false;
  if (!upload((void**)&E->d_items, items.data(), items.size() * sizeof(PItem))) return false;
  if (!upload((void**)&E->d_recs, recs.data(), recs.size() * sizeof(uint32_t))) return false;
  LE_CK(cudaMalloc(&E->d_norms, (size_t)(2 * L + 1) * E->dim * 4));
  for (int l = 0; l < L; ++l) {
    LE_CK(cudaMemcpy(E->d_norms + (size_t)(2 * l) * E->dim, E->L[l].in_norm, E->dim * 4, cudaMemcpyDeviceToDevice));
    LE_CK(cudaMemcpy(E->d_norms + (size_t)(2 * l + 1) * E->dim, E->L[l].post_norm, E->dim * 4,
                     cudaMemcpyDeviceToDevice));
  }
  LE_CK(cudaMemcpy(E->d_norms + (size_t)(2 * L) * E->dim, E->final_norm, E->dim * 4, cudaMemcpyDeviceToDevice));
  const size_t n_tagged = (size_t)E->dim + (E->dim + 2 * E->kv_dim) + E->dim + E->ffn;
  LE_CK(cudaMalloc(&E->d_tagged, n_tagged * sizeof(unsigned long long)));
  LE_CK(cudaMemset(E->d_tagged, 0, n_tagged * sizeof(unsigned long long)));  // tag 0 is never valid
  E->d_ctrl = reinterpret_cast<PCtrl*>(E->ctrl_block);  // am_result follows it (greedy())
  LE_CK(cudaMemset(E->d_ctrl, 0, sizeof(PCtrl)));
  // mapped completion words (greedy()); without them sample() reads the result with a copy
  uint32_t* d_done = nullptr;
  if (cudaHostAlloc(&E->h_done, 64, cudaHostAllocMapped) == cudaSuccess) {
    std::memset(E->h_done, 0, 64);
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_done), E->h_done, 0) != cudaSuccess) d_done = nullptr;
  } else {
    E->h_done = nullptr;
  }
  cudaGetLastError();  // a failed mapping only disables the fast path
  PArgs& A = E->pargs;
  A.arena = E->rec_arena;
  A.sched = E->d_sched; A.segs = E->d_segs; A.items = E->d_items; A.recs = E->d_recs;
  A.norms = E->d_norms;
  A.rope_cos = E->rope_cos; A.rope_sin = E->rope_sin;
  A.x = E->d_tagged;
  A.qkv = A.x + E->dim;
  A.attn = A.qkv + E->dim + 2 * E->kv_dim;
  A.act = A.attn + E->dim;
  A.logits = E->logits;
  A.kcache = E->kcache; A.vcache = E->vcache;
  A.ctrl = E->d_ctrl;
  A.token_log = E->token_log; A.am_result = E->am_result;
  A.lm_rec_base = (unsigned long long)lm_base * kRecBytes;
  A.wait_ns = kWaitNs;
  A.layers = L; A.dim = (int)E->dim; A.ffn = (int)E->ffn; A.vocab = (int)E->vocab;
  A.heads = (int)E->heads; A.kv_heads = (int)E->kv_heads; A.max_seq = E->max_seq;
  A.n_lm_ctas = n_lm_ctas;
  A.n_tokens = 1; A.do_logits = 1;
  A.token0 = 0; A.pos0 = 0;
  A.host_done = d_done; A.seq = 0;
  A.expire_where = 0;
  E->p_grid = G;
  LE_CK(cudaStreamSynchronize(E->stream));
  E->persist = true;
  return true;
}

// Every change of the greedy-result state goes through here: `persist` says that am_result[0]
// (and the mapped h_done words) hold the greedy id of the newest persistent launch.
static void set_argmax(Engine* E, bool valid, bool persist = false) {
  E->argmax_valid = valid;
  E->argmax_persist = valid && persist;
}

// One cooperative launch of n_tokens steps on slot 0 from (token, pos); the token and position
// are kernel arguments, so a step needs no parameter copy.
static bool launch_persistent(Engine* E, int n_tokens, bool logits, int32_t token, int32_t pos) {
  PArgs A = E->pargs;
  A.n_tokens = n_tokens;
  A.do_logits = logits ? 1 : 0;
  A.token0 = token;
  A.pos0 = pos;
  A.seq = ++E->persist_seq;
  if (logits) E->persist_seq_logits = A.seq;
  void* args[] = {&A};
  const void* fn = A.trace ? (const void*)k_decode_persistent<true> : (const void*)k_decode_persistent<false>;
  LE_CK(cudaLaunchCooperativeKernel(fn, dim3(E->p_grid), dim3(kPThreads), args,
                                    persistent_smem(), E->stream));
  return true;
}


// ---------------------------------------------------------------------------------------------
// Token-batched path: batched decode over sequence slots and chunked prefill, with every weight
// GEMM on the tensor cores (tc_gemm.cuh).
// ---------------------------------------------------------------------------------------------
static bool tc_supported(const Engine* E) {
  const char* v = getenv("LLAMA_B200_BATCHED");
  if (v && std::strcmp(v, "0") == 0) return false;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, E->device) != cudaSuccess || prop.major != 10) return false;
  return E->dim % 2048 == 0 && E->ffn % 2048 == 0 && E->heads == 4 * E->kv_heads;
}

static bool init_tc(Engine* E) {
  if (!tc_supported(E)) return true;
  using namespace tc;
  const int dim = (int)E->dim, ffn = (int)E->ffn, kvd = (int)E->kv_dim, L = (int)E->layers;
  // rows per batched step: the sequence slots, and at least one prefill chunk
  // ($LLAMA_B200_PREFILL_CHUNK tokens, default 2048: a 2048-id prompt in one chunk measured 7 %
  // faster than two chunks of 1024 and 22 % faster than four of 512)
  int chunk = 2048;
  if (const char* c = getenv("LLAMA_B200_PREFILL_CHUNK")) chunk = std::max(kTok, std::min(8192, atoi(c)));
  chunk = (chunk + kTok - 1) / kTok * kTok;
  E->tc_T = std::max(chunk, (E->max_batch + kTok - 1) / kTok * kTok);
  const int T = E->tc_T;
  // ---- weight records ----
  const int kb_d = dim / 128, kb_f = ffn / 128;
  const int t_qkv = (dim + 2 * kvd + kM - 1) / kM, t_o = dim / kM, t_gu = ffn / 64, t_d = dim / kM;
  const int t_lm = ((int)E->vocab + kM - 1) / kM;
  const size_t per_layer = (size_t)(t_qkv + t_o + t_gu) * kb_d + (size_t)t_d * kb_f;
  const size_t total = (per_layer * L + (size_t)t_lm * kb_d) * tc::kRecBytes;
  LE_CK(cudaMalloc(&E->tc_arena, total));
  LE_CK(cudaMemsetAsync(E->tc_arena, 0, total, E->stream));
  size_t off = 0;
  auto take = [&](int tiles, int kb) {
    TcMat m;
    m.recs = E->tc_arena + off;
    m.tiles = tiles;
    m.kb = kb;
    off += (size_t)tiles * kb * tc::kRecBytes;
    return m;
  };
  auto repack = [&](const QMat& W, const TcMat& M, int row0, int G, int o, int stride = 1) -> bool {
    k_tc_repack<<<E->num_sms * 8, 256, 0, E->stream>>>(W, const_cast<uint8_t*>(M.recs), row0, G, o, stride);
    LE_CK(cudaGetLastError());
    return true;
  };
  E->tcl.resize(L);
  for (int l = 0; l < L; ++l) {
    TcLayer& Y = E->tcl[l];
    const DevLayer& D = E->L[l];
    Y.qkv = take(t_qkv, kb_d);
    Y.o = take(t_o, kb_d);
    Y.gu = take(t_gu, kb_d);
    Y.d = take(t_d, kb_f);
    if (!repack(D.q, Y.qkv, 0, kM, 0) || !repack(D.k, Y.qkv, dim, kM, 0) || !repack(D.v, Y.qkv, dim + kvd, kM, 0))
      return false;
    if (!repack(D.o, Y.o, 0, kM, 0)) return false;
    if (!repack(D.g, Y.gu, 0, 64, 0, 2) || !repack(D.u, Y.gu, 0, 64, 1, 2)) return false;
    if (!repack(D.d, Y.d, 0, kM, 0)) return false;
  }
  E->tc_lm = take(t_lm, kb_d);
  if (!repack(E->lm_head, E->tc_lm, 0, kM, 0)) return false;
  // ---- activations ----
  const size_t tiles_T = (size_t)T / kTok;
  LE_CK(cudaMalloc(&E->img_d, tiles_T * kb_d * kImgBytes));
  LE_CK(cudaMalloc(&E->img_f, tiles_T * kb_f * kImgBytes));
  LE_CK(cudaMemsetAsync(E->img_d, 0, tiles_T * kb_d * kImgBytes, E->stream));
  LE_CK(cudaMemsetAsync(E->img_f, 0, tiles_T * kb_f * kImgBytes, E->stream));
  LE_CK(cudaMalloc(&E->t_x, (size_t)T * dim * 4));
  LE_CK(cudaMalloc(&E->t_q, (size_t)T * dim * 4));
  LE_CK(cudaMalloc(&E->t_attn, (size_t)T * dim * 4));
  LE_CK(cudaMalloc(&E->t_qkv, (size_t)kTcMaxSplits * T * (dim + 2 * kvd) * 4));
  LE_CK(cudaMalloc(&E->t_gu, (size_t)T * ffn * 4));
  LE_CK(cudaMalloc(&E->t_part, (size_t)kTcMaxSplits * T * dim * 4));
  LE_CK(cudaMalloc(&E->t_attn_part, (size_t)T * E->kv_heads * kAttnMaxSplits * kAttnPart * 4));
  E->kv_img_tiles = (E->max_seq + attn::kKeys - 1) / attn::kKeys;
  LE_CK(cudaMalloc(&E->kv_img, (size_t)E->kv_heads * E->kv_img_tiles * attn::kTileBytes));
  LE_CK(cudaMalloc(&E->t_idx, (size_t)3 * T * 4));
  LE_CK(cudaMallocHost(&E->h_idx, (size_t)3 * T * 4));
  LE_CK(cudaEventCreateWithFlags(&E->idx_ev, cudaEventDisableTiming));
  E->tc_am_parts = std::min<int>(64, ((int)E->vocab + 4 * 256 - 1) / (4 * 256));
  LE_CK(cudaMalloc(&E->t_am, (size_t)T * E->tc_am_parts * sizeof(ArgmaxPart)));
  LE_CK(cudaMalloc(&E->tc_err, 16));
  LE_CK(cudaMemsetAsync(E->tc_err, 0, 16, E->stream));
  LE_CK(cudaFuncSetAttribute(k_tc_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<1>::kSmemBytes));
  LE_CK(cudaFuncSetAttribute(k_tc_gemm<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<2>::kSmemBytes));
  LE_CK(cudaFuncSetAttribute(k_attn_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
  LE_CK(cudaFuncSetAttribute(k_attn_prefill_tc5, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::kSmemBytes));
  int per_sm = 0, per_sm2 = 0;
  LE_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_tc_gemm<1>, Geo<1>::kThreads, Geo<1>::kSmemBytes));
  LE_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm2, k_tc_gemm<2>, Geo<2>::kThreads, Geo<2>::kSmemBytes));
  if (std::min(per_sm, per_sm2) < 1) {
    E->err = "tensor-core GEMM declined: 0 resident CTAs per SM";
    return true;
  }
  LE_CK(cudaStreamSynchronize(E->stream));
  E->tc = true;
  return true;
}

// Number of K splits for a GEMM whose tiles x token groups alone would leave SMs idle.
static int tc_splits(int num_sms, int tiles, int kb, int tok_groups) {
  const int base = tiles * tok_groups;
  if (base >= num_sms) {
    // enough units for every SM: split K in two only for long K (the down projection), where the
    // fuller last wave outweighs the extra partial plane (units per wave-slot: busy fraction)
    auto busy = [&](int s) {
      const int u = base * s, waves = (u + num_sms - 1) / num_sms;
      return (double)u / (double)(waves * num_sms);
    };
    return (kb >= 32 && busy(2) > busy(1) + 0.05) ? 2 : 1;
  }
  int s = std::min(kTcMaxSplits, num_sms / base);
  s = std::min(s, std::max(1, kb / 2));
  return std::max(1, s);
}

// Unit form and K splits of one tensor-core GEMM launch: P = 1 (64-token units) or 2 (128-token
// units over two image tiles), whichever gives the shorter estimate = K blocks of the busiest CTA
// x the form's block period (768 and 1056 ns, measured by the per-block pipeline trace at 64 and
// 128 tokens).  Two-tile units halve the issuer's cost per token but also the unit count, so small
// steps keep one-tile units; one image tile cannot pair.  splits_req > 0 fixes the splits.
struct TcPlan {
  int P = 1, groups = 1, splits = 1, kb_split = 1;
};
static TcPlan tc_plan(int num_sms, int tiles, int kb, int img_tiles, int splits_req) {
  static constexpr double kBlockNs[3] = {0.0, 768.0, 1056.0};
  TcPlan best;
  double best_ns = 0.0;
  for (int P = 1; P <= 2; ++P) {
    if (P == 2 && (img_tiles < 2 || !tc_pair_enabled())) continue;
    TcPlan c;
    c.P = P;
    c.groups = (img_tiles + P - 1) / P;
    const int want = splits_req > 0 ? splits_req : tc_splits(num_sms, tiles, kb, c.groups);
    c.kb_split = (kb + want - 1) / want;
    c.splits = (kb + c.kb_split - 1) / c.kb_split;
    const long long units = (long long)tiles * c.groups * c.splits;
    const long long grid = std::min<long long>(units, num_sms);
    const double ns = (double)((units + grid - 1) / grid) * c.kb_split * kBlockNs[P];
    if (P == 1 || ns < best_ns) {
      best = c;
      best_ns = ns;
    }
  }
  return best;
}

// Launch with programmatic stream serialisation: the kernel may be scheduled while the previous
// kernel of the stream is still finishing (it waits for it with griddepcontrol.wait before
// touching any activation), which hides the launch gap between the dependent kernels of a step.
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Launches one tensor-core GEMM over T token rows of `img`; returns the number of K splits used
// (splits < 0: chosen for the shape; the unit form is chosen by tc_plan).
static int tc_launch(Engine* E, const TcMat& W, const uint8_t* img, int T, int splits, tc::Args A) {
  A.recs = W.recs;
  A.img = img;
  A.tiles = W.tiles;
  A.kb_total = W.kb;
  A.img_tiles = (T + tc::kTok - 1) / tc::kTok;
  const TcPlan pl = tc_plan(E->num_sms, W.tiles, W.kb, A.img_tiles, splits);
  const int P = pl.P;
  A.tok_tiles = pl.groups;
  A.T = T;
  A.kb_split = pl.kb_split;
  A.splits = pl.splits;
  A.error = E->tc_err;
  A.wait_ns = E->tc_wait_ns;
  A.expire = E->tc_expire;
  const int units = A.tiles * A.tok_tiles * A.splits;
  if (P == 2)
    launch_pdl(tc::k_tc_gemm<2>, dim3(std::min(units, E->num_sms)), dim3(tc::Geo<2>::kThreads), tc::Geo<2>::kSmemBytes,
               E->stream, A);
  else
    launch_pdl(tc::k_tc_gemm<1>, dim3(std::min(units, E->num_sms)), dim3(tc::Geo<1>::kThreads), tc::Geo<1>::kSmemBytes,
               E->stream, A);
  return A.splits;
}

// Copies (token, position, slot) of n rows to the device (one H2D copy from pinned memory).
static bool tc_upload_rows(Engine* E, const int32_t* tok, const int32_t* pos, const int32_t* slot, int n) {
  if (E->idx_pending) LE_CK(cudaEventSynchronize(E->idx_ev));
  for (int i = 0; i < n; ++i) {
    int32_t t = tok[i];
    if (t < 0 || t >= (int32_t)E->vocab) t = 0;  // src/llama_engine.cpp:937
    E->h_idx[i] = t;
    E->h_idx[n + i] = pos[i];
    E->h_idx[2 * n + i] = slot[i];
  }
  LE_CK(cudaMemcpyAsync(E->t_idx, E->h_idx, (size_t)3 * n * 4, cudaMemcpyHostToDevice, E->stream));
  LE_CK(cudaEventRecord(E->idx_ev, E->stream));
  E->idx_pending = true;
  return true;
}

// Position-range splits of decode attention (each range >= 1024 positions); one formula for the
// step and for its graph-cache key.  (Also limiting the splits by rows x kv heads measured the
// same at 256 rows.)
static int attn_splits_for(int max_pos) { return std::max(1, std::min(kAttnMaxSplits, (max_pos + 1) / 1024)); }

// One forward step of n rows (rows already uploaded).  Logits and greedy ids are produced for
// rows [lrow0, lrow0 + nlog) into logits rows 0..nlog-1 and am_result[0..nlog-1].
// With prefill_p0 >= 0 the rows are consecutive positions prefill_p0 .. of slot 0 (a prefill
// chunk) and attention runs query-tiled.
// fold: every row is a different slot, so no row reads another row's new k / v; RoPE and the
// KV append then run inside the decode attention kernel.
static bool tc_step(Engine* E, int n, int lrow0, int nlog, int max_pos, int prefill_p0 = -1,
                    float* logits_out = nullptr, bool fold = false) {
  float* const lg_out = logits_out ? logits_out : E->logits;
  using namespace tc;
  const int dim = (int)E->dim, ffn = (int)E->ffn, kvd = (int)E->kv_dim;
  const size_t layer_stride = (size_t)E->max_seq * kvd;
  const size_t slot_stride = (size_t)E->layers * layer_stride;
  const size_t part_stride = (size_t)E->tc_T * dim;
  const int32_t* tok = E->t_idx;
  const int32_t* pos = E->t_idx + n;
  const int32_t* slot = E->t_idx + 2 * n;
  const int attn_splits = attn_splits_for(max_pos);
  cudaStream_t s = E->stream;
  auto rows = [&](float* out, int ldo, int N, size_t split_stride) {
    Args A{};
    A.out = out;
    A.ldo = ldo;
    A.N = N;
    A.split_stride = split_stride;
    return A;
  };
  // staging with every split-K plane's loads at once for steps of up to one row per SM (decode
  // batches, where the step is latency-bound), three at a time for larger steps (occupancy)
  auto stage_fn = n <= E->num_sms ? k_tc_stage<true> : k_tc_stage<false>;
  k_embed_batch<<<n, 256, 0, s>>>(E->lm_head, tok, E->t_x, dim);
  int d_splits = 0;
  for (uint32_t l = 0; l < E->layers; ++l) {
    const TcLayer& Y = E->tcl[l];
    const DevLayer& D = E->L[l];
    float* kc = E->kcache + l * layer_stride;
    float* vc = E->vcache + l * layer_stride;
    launch_pdl(stage_fn, dim3(n), dim3(256), 0, s, E->t_x, dim, E->t_part, d_splits, part_stride, D.in_norm, dim,
               E->img_d);
    const size_t qkv_stride = (size_t)E->tc_T * (dim + 2 * kvd);
    const int sq = tc_launch(E, Y.qkv, E->img_d, n, -1,
                             rows(E->t_qkv, dim + 2 * kvd, dim + 2 * kvd, qkv_stride));
    if (prefill_p0 >= 0 || !fold)
      launch_pdl(k_rope_append, dim3(n), dim3(256), 0, s, E->t_qkv, sq, qkv_stride,
                 dim, kvd, pos, slot, E->rope_cos, E->rope_sin, E->t_q, kc, vc, slot_stride);
    if (prefill_p0 >= 0) {
      const int p_last = prefill_p0 + n - 1;
      launch_pdl(k_kv_tiles, dim3(E->kv_heads, p_last / attn::kKeys + 1), dim3(128), 0, s, kc, vc, kvd, p_last,
                 E->kv_img, E->kv_img_tiles);
      launch_pdl(k_attn_prefill_tc5, dim3(E->kv_heads, (n + attn::kQ - 1) / attn::kQ), dim3(128),
                 (size_t)attn::kSmemBytes, s, E->t_q, dim, E->kv_img, E->kv_img_tiles, prefill_p0, n, E->t_attn,
                 E->tc_err, E->attn_wait_ns, E->attn_expire);
    } else {
      // decode rows: RoPE and the KV append run inside the attention kernel
      // without position splits the attention kernel writes the o-proj input image itself
      launch_pdl(k_attn_batch, dim3(n, E->kv_heads, attn_splits), dim3(128), kAttnSmem, s, E->t_q, dim, kc, vc,
                 slot_stride, kvd, pos, slot, E->t_attn, E->t_attn_part, fold ? E->t_qkv : nullptr, sq, qkv_stride,
                 E->rope_cos, E->rope_sin, attn_splits == 1 ? E->img_d : nullptr);
      if (attn_splits > 1)
        launch_pdl(k_attn_combine, dim3(n), dim3(256), 0, s, E->t_attn_part, (int)E->kv_heads, attn_splits, dim,
                   E->t_attn);
    }
    if (prefill_p0 >= 0 || attn_splits > 1)
      launch_pdl(stage_fn, dim3(n, dim / 2048), dim3(256), 0, s, E->t_attn, dim, nullptr, 0, 0, nullptr, dim,
                 E->img_d);
    const int so = tc_launch(E, Y.o, E->img_d, n, -1, rows(E->t_part, dim, dim, part_stride));
    launch_pdl(stage_fn, dim3(n), dim3(256), 0, s, E->t_x, dim, E->t_part, so, part_stride, D.post_norm, dim,
               E->img_d);
    Args Agu = rows(E->t_gu, ffn, ffn, 0);
    Agu.swiglu = 1;
    tc_launch(E, Y.gu, E->img_d, n, 1, Agu);
    launch_pdl(stage_fn, dim3(n, ffn / 2048), dim3(256), 0, s, E->t_gu, ffn, nullptr, 0, 0, nullptr, ffn,
               E->img_f);
    d_splits = tc_launch(E, Y.d, E->img_f, n, -1, rows(E->t_part, dim, dim, part_stride));
  }
  if (nlog > 0) {
    launch_pdl(stage_fn, dim3(nlog), dim3(256), 0, s, E->t_x + (size_t)lrow0 * dim, dim,
               E->t_part + (size_t)lrow0 * dim, d_splits, part_stride, E->final_norm, dim, E->img_d);
    tc_launch(E, E->tc_lm, E->img_d, nlog, 1, rows(lg_out, (int)E->vocab, (int)E->vocab, 0));
    if (!logits_out) {
      launch_pdl(k_argmax_rows_batch, dim3(E->tc_am_parts, nlog), dim3(256), 0, s, E->logits, (int)E->vocab,
                 (size_t)E->vocab, E->t_am);
      launch_pdl(k_argmax_finish_batch, dim3(nlog), dim3(256), 0, s, E->t_am, E->tc_am_parts, E->am_result);
    }
  }
  LE_CK(cudaGetLastError());
  E->tc_dirty = true;
  return true;
}

// A decode step (rows already uploaded) through a cached CUDA graph of tc_step's launches.
static bool tc_step_graph(Engine* E, int n, int nlog, int max_pos, bool fold) {
  const int splits = attn_splits_for(max_pos);
  for (const auto& g : E->tc_graphs)
    if (g.n == n && g.nlog == nlog && g.splits == splits && g.fold == fold) {
      LE_CK(cudaGraphLaunch(g.exec, E->stream));
      E->tc_dirty = true;
      return true;
    }
  if (E->tc_graphs.size() >= 64) return tc_step(E, n, 0, nlog, max_pos, -1, nullptr, fold);  // launch directly
  LE_CK(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  const bool ok = tc_step(E, n, 0, nlog, max_pos, -1, nullptr, fold);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(E->stream, &graph);
  if (!ok || ce != cudaSuccess || graph == nullptr) {
    if (graph) cudaGraphDestroy(graph);
    E->err = std::string("batched step capture failed: ") + cudaGetErrorString(ce);
    return false;
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) { E->err = cudaGetErrorString(ie); return false; }
  E->tc_graphs.push_back({n, nlog, splits, fold, exec});
  LE_CK(cudaGraphLaunch(exec, E->stream));
  return true;
}

// Chunked prefill of `count` tokens of slot 0 at positions start .. start+count-1.
static bool tc_prefill(Engine* E, const int32_t* ids, size_t count, size_t start, bool last_logits) {
  std::vector<int32_t> pos(E->tc_T), slot(E->tc_T, 0);
  for (size_t c0 = 0; c0 < count; c0 += (size_t)E->tc_T) {
    const int n = (int)std::min<size_t>((size_t)E->tc_T, count - c0);
    for (int i = 0; i < n; ++i) pos[i] = (int32_t)(start + c0 + i);
    if (!tc_upload_rows(E, ids + c0, pos.data(), slot.data(), n)) return false;
    const bool lg = last_logits && c0 + n == count;
    if (!tc_step(E, n, n - 1, lg ? 1 : 0, (int)(start + c0) + n - 1, (int)(start + c0))) return false;
  }
  return true;
}

static bool persistent_ok(Engine* E);
// Synchronises the stream and reports a device error recorded by the last steps.
static bool sync_ok(Engine* E) {
  if (E->persist || E->tc) return persistent_ok(E);
  const cudaError_t ce = cudaStreamSynchronize(E->stream);
  if (ce != cudaSuccess) { E->err = cudaGetErrorString(ce); return false; }
  return true;
}

// Device error words of the persistent kernel and of the tensor-core GEMM: the copies are queued
// behind the work (the GEMM's only when a batched step ran since it was last read) and checked
// after the caller's synchronisation, so that a token id and its status cost one wait.
static bool enqueue_status(Engine* E) {
  if (E->persist)
    LE_CK(cudaMemcpyAsync(E->h_err, &E->d_ctrl->error, 2 * sizeof(uint32_t), cudaMemcpyDeviceToHost, E->stream));
  if (E->tc && E->tc_dirty)
    LE_CK(cudaMemcpyAsync(E->h_err + 2, E->tc_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, E->stream));
  return true;
}
static bool check_status(Engine* E) {
  const bool tc_read = E->tc && E->tc_dirty;
  E->tc_dirty = false;
  if (E->persist && E->h_err[0] != 0) {
    E->err = "persistent decode kernel: a dependency wait timed out (code " + std::to_string(E->h_err[1]) + ")";
    return false;
  }
  if (tc_read && E->h_err[2] != 0) {
    E->err = (E->h_err[2] == (uint32_t)kExpireAttn ? "prefill attention (tensor cores): a wait timed out (code "
                                                    : "tensor-core GEMM: a pipeline wait timed out (code ") +
             std::to_string(E->h_err[2]) + ")";
    E->tc_dirty = true;  // keep reporting it
    return false;
  }
  return true;
}

static bool persistent_ok(Engine* E) {
  if (!E->persist && !E->tc) return true;
  if (!enqueue_status(E)) return false;
  LE_CK(cudaStreamSynchronize(E->stream));
  return check_status(E);
}

// RoPE tables [n_pos][32] (cos, sin).  The default is the reference's table: theta_i =
// powf(500000, -2i/64), cos/sin(pos * theta_i) in float with the same libm calls
// (src/llama_engine.cpp:908-917), so the table is bit-identical.  With factor > 0 the
// frequencies are first rescaled the "llama3" way (the rope_scaling of the reference's
// models/config.json:26-32, applied by its Hugging Face path chat.py:42 but not by the C++
// engine): with wavelength w_i = 2 pi / theta_i, low = original / low_freq_factor and
// high = original / high_freq_factor, theta_i is kept when w_i < high, divided by factor when
// w_i > low, and in between blended as (1 - s) theta_i / factor + s theta_i with
// s = (original / w_i - low_freq_factor) / (high_freq_factor - low_freq_factor).
struct RopeScaling {
  float factor = 0.0f;  // <= 0: the reference's unscaled table
  float low_freq_factor = 1.0f, high_freq_factor = 4.0f;
  int original_max_position = 8192;
};

static void build_rope_table(const RopeScaling& rs, int n_pos, std::vector<float>& cs, std::vector<float>& sn) {
  const size_t hd2 = LE_HEAD_DIM / 2;
  float theta[LE_HEAD_DIM / 2];
  for (size_t i = 0; i < hd2; ++i) {
    theta[i] = std::pow(500000.0f, -2.0f * static_cast<float>(i) / static_cast<float>(LE_HEAD_DIM));
    if (rs.factor > 0.0f) {
      const double pi = 3.14159265358979323846, t = theta[i];
      const double w = 2.0 * pi / t, orig = rs.original_max_position;
      const double low = orig / rs.low_freq_factor, high = orig / rs.high_freq_factor;
      double v = t;
      if (w > low) {
        v = t / rs.factor;
      } else if (w >= high) {
        const double sm = (orig / w - rs.low_freq_factor) / (rs.high_freq_factor - rs.low_freq_factor);
        v = (1.0 - sm) * t / rs.factor + sm * t;
      }
      theta[i] = static_cast<float>(v);
    }
  }
  cs.assign((size_t)n_pos * hd2, 0.0f);
  sn.assign((size_t)n_pos * hd2, 0.0f);
  for (size_t pos = 0; pos < (size_t)n_pos; ++pos) {
    for (size_t i = 0; i < hd2; ++i) {
      cs[pos * hd2 + i] = std::cos(static_cast<float>(pos) * theta[i]);
      sn[pos * hd2 + i] = std::sin(static_cast<float>(pos) * theta[i]);
    }
  }
}

static bool init_device(Engine* E, const uint8_t* base, const ParsedFile& P) {
  LE_CK(cudaSetDevice(E->device));
  LE_CK(cudaDeviceGetAttribute(&E->num_sms, cudaDevAttrMultiProcessorCount, E->device));
  LE_CK(cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking));
  E->layers = P.layers; E->dim = P.dim; E->ffn = P.ffn; E->vocab = P.vocab;
  E->heads = P.heads; E->kv_heads = P.kv_heads; E->kv_dim = P.kv_heads * LE_HEAD_DIM;

  // ---- weight arena: every array 256-byte aligned ----
  auto mat_bytes = [](const FileMatrix& m) {
    return align_up((size_t)m.nb * 64, 256) + 2 * align_up((size_t)m.nb * 2, 256);
  };
  size_t total = align_up((size_t)P.dim * 4, 256);
  for (const auto& Ly : P.L) {
    total += 2 * align_up((size_t)P.dim * 4, 256);
    for (int i = 0; i < 7; ++i) total += mat_bytes(Ly.m[i]);
  }
  total += mat_bytes(P.lm_head);
  E->arena_bytes = total;
  LE_CK(cudaMalloc(&E->arena, total));
  size_t off = 0;
  auto put = [&](size_t n) -> uint8_t* {
    uint8_t* dst = E->arena + off;
    off += align_up(n, 256);
    return dst;
  };
  // Copy in large pieces straight from the mapping.
  std::vector<std::pair<uint8_t*, std::pair<size_t, size_t>>> copies;
  auto place = [&](size_t src_off, size_t n) -> uint8_t* {
    uint8_t* d = put(n);
    copies.push_back({d, {src_off, n}});
    return d;
  };
  auto place_mat = [&](const FileMatrix& m) -> QMat {
    QMat q;
    q.N = (int)m.N; q.K = (int)m.K;
    q.nib = place(m.nib_off, (size_t)m.nb * 64);
    q.step = reinterpret_cast<const uint16_t*>(place(m.step_off, (size_t)m.nb * 2));
    q.mn = reinterpret_cast<const uint16_t*>(place(m.min_off, (size_t)m.nb * 2));
    return q;
  };
  E->final_norm = reinterpret_cast<const float*>(place(P.final_norm_off, (size_t)P.dim * 4));
  E->L.resize(P.layers);
  for (uint32_t l = 0; l < P.layers; ++l) {
    DevLayer& D = E->L[l];
    D.in_norm = reinterpret_cast<const float*>(place(P.L[l].in_norm_off, (size_t)P.dim * 4));
    D.post_norm = reinterpret_cast<const float*>(place(P.L[l].post_norm_off, (size_t)P.dim * 4));
    D.q = place_mat(P.L[l].m[0]); D.k = place_mat(P.L[l].m[1]); D.v = place_mat(P.L[l].m[2]);
    D.o = place_mat(P.L[l].m[3]); D.g = place_mat(P.L[l].m[4]); D.u = place_mat(P.L[l].m[5]);
    D.d = place_mat(P.L[l].m[6]);
  }
  E->lm_head = place_mat(P.lm_head);
  for (auto& c : copies) LE_CK(cudaMemcpy(c.first, base + c.second.first, c.second.second, cudaMemcpyHostToDevice));

  // ---- RoPE table on the host, same float calls as src/llama_engine.cpp:911-917 ----
  {
    std::vector<float> cs, sn;
    build_rope_table(RopeScaling{}, LE_MAX_SEQ_LEN, cs, sn);
    LE_CK(cudaMalloc(&E->rope_cos, cs.size() * 4));
    LE_CK(cudaMalloc(&E->rope_sin, sn.size() * 4));
    LE_CK(cudaMemcpy(E->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    LE_CK(cudaMemcpy(E->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }

  // ---- KV caches and activations ----
  const size_t kv_elems = (size_t)E->max_batch * E->layers * E->max_seq * E->kv_dim;
  LE_CK(cudaMalloc(&E->kcache, kv_elems * 4));
  LE_CK(cudaMalloc(&E->vcache, kv_elems * 4));
  LE_CK(cudaMemsetAsync(E->kcache, 0, kv_elems * 4, E->stream));
  LE_CK(cudaMemsetAsync(E->vcache, 0, kv_elems * 4, E->stream));
  const size_t B = (size_t)E->max_batch;
  E->lm_grid = std::min<int>((int)((E->vocab / 2 + kWarps - 1) / kWarps), E->num_sms * 8);
  LE_CK(cudaMalloc(&E->x, B * E->dim * 4));
  LE_CK(cudaMalloc(&E->qkv, B * (E->dim + 2 * E->kv_dim) * 4));
  LE_CK(cudaMalloc(&E->attn, B * E->dim * 4));
  LE_CK(cudaMalloc(&E->act, B * E->ffn * 4));
  LE_CK(cudaMalloc(&E->logits, B * E->vocab * 4));
  LE_CK(cudaMemsetAsync(E->logits, 0, B * E->vocab * 4, E->stream));
  LE_CK(cudaMalloc(&E->emb, (size_t)E->dim * 4));
  LE_CK(cudaMalloc(&E->red, 2048 * 4));
  LE_CK(cudaMalloc(&E->d_misc, 16 * 4));
  LE_CK(cudaMalloc(&E->part, B * E->lm_grid * sizeof(ArgmaxPart)));
  // the persistent kernel's control words and the greedy results in one allocation, am_result
  // right after PCtrl: greedy() reads the error words and am_result[0] with one copy
  LE_CK(cudaMalloc(&E->ctrl_block, sizeof(PCtrl) + B * 4));
  LE_CK(cudaMemsetAsync(E->ctrl_block, 0, sizeof(PCtrl) + B * 4, E->stream));
  E->am_result = reinterpret_cast<int32_t*>(E->ctrl_block + sizeof(PCtrl));
  LE_CK(cudaMalloc(&E->token_log, (size_t)LE_MAX_SEQ_LEN * 4));
  LE_CK(cudaMalloc(&E->d_params, B * sizeof(StepParams)));
  LE_CK(cudaMemsetAsync(E->d_params, 0, B * sizeof(StepParams), E->stream));
  LE_CK(cudaMallocHost(&E->h_ring, kRing * sizeof(StepParams)));
  for (int i = 0; i < kRing; ++i) LE_CK(cudaEventCreateWithFlags(&E->ring_ev[i], cudaEventDisableTiming));
  LE_CK(cudaMallocHost(&E->h_logits, B * E->vocab * 4));
  LE_CK(cudaMallocHost(&E->h_small, (size_t)LE_MAX_SEQ_LEN * 4));
  LE_CK(cudaMallocHost(&E->h_err, 4 * sizeof(uint32_t)));
  for (int i = 0; i < 4; ++i) E->h_err[i] = 0;
  if (!set_smem_attrs(E)) return false;

  // ---- graphs ----
  if (!capture(E, row_buffers(E, 0, 0, false, 0), &E->g_fwd[0])) return false;
  if (!capture(E, row_buffers(E, 0, 0, true, 0), &E->g_fwd[1])) return false;
  if (!capture(E, row_buffers(E, 0, 0, true, 1), &E->g_gen)) return false;
  LE_CK(cudaStreamSynchronize(E->stream));
  if (E->tp_world > 1) return true;  // the tensor-parallel engine runs its own graph (init_tp)
  if (!init_persistent(E)) return false;
  if (!init_tc(E)) return false;
  return true;
}

static void destroy_tp(Engine* E);
static void destroy(Engine* E) {
  if (!E) return;
  DeviceGuard dg(E->device);
  if (E->stream) cudaStreamSynchronize(E->stream);
  destroy_tp(E);
  for (auto& g : E->g_fwd) if (g) cudaGraphExecDestroy(g);
  for (auto& g : E->tc_graphs) if (g.exec) cudaGraphExecDestroy(g.exec);
  if (E->g_gen) cudaGraphExecDestroy(E->g_gen);
  for (auto& ev : E->ring_ev) if (ev) cudaEventDestroy(ev);
  void* pdev[] = {E->d_trace, E->rec_arena, E->d_sched, E->d_segs, E->d_items, E->d_recs, (void*)E->d_norms, E->d_tagged};
  for (void* p : pdev) if (p) cudaFree(p);
  if (E->h_err) cudaFreeHost(E->h_err);
  if (E->h_done) cudaFreeHost(E->h_done);
  void* tdev[] = {E->tc_arena, E->img_d, E->img_f, E->t_x, E->t_q, E->t_attn, E->t_qkv, E->t_gu, E->t_part,
                  E->t_idx, E->t_am, E->tc_err, E->t_attn_part, E->kv_img, E->sc_logits, E->sc_target, E->sc_lp,
                  E->sc_greedy};
  for (void* p : tdev) if (p) cudaFree(p);
  if (E->h_idx) cudaFreeHost(E->h_idx);
  if (E->idx_ev) cudaEventDestroy(E->idx_ev);
  void* dev_ptrs[] = {E->arena, E->rope_cos, E->rope_sin, E->kcache, E->vcache, E->x, E->qkv, E->attn,
                      E->act, E->logits, E->emb, E->red, E->d_misc, E->part, E->ctrl_block, E->token_log, E->d_params};
  for (void* p : dev_ptrs) if (p) cudaFree(p);
  if (E->h_ring) cudaFreeHost(E->h_ring);
  if (E->h_logits) cudaFreeHost(E->h_logits);
  if (E->h_small) cudaFreeHost(E->h_small);
  if (E->stream) cudaStreamDestroy(E->stream);
  delete E;
}

static bool init_tp(Engine* E, const ncclUniqueId& id);
static Engine* create(const char* path, int device, int max_batch, int max_seq, int tp_rank = 0, int tp_world = 1,
                      const ncclUniqueId* tp_id = nullptr) {
  if (!path) { set_create_error("model path is NULL"); return nullptr; }
  if (max_batch < 1 || max_batch > 4096) { set_create_error("max_batch out of range"); return nullptr; }
  if (max_seq == 0) max_seq = LE_MAX_SEQ_LEN;
  if (max_seq < 1 || max_seq > LE_MAX_SEQ_LEN) { set_create_error("max_seq_len out of range"); return nullptr; }
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) { set_create_error(std::string("cannot open ") + path); return nullptr; }
  struct stat sb;
  if (fstat(fd, &sb) != 0) { ::close(fd); set_create_error("fstat failed"); return nullptr; }
  const size_t size = (size_t)sb.st_size;
  void* map = size ? mmap(nullptr, size, PROT_READ, MAP_SHARED, fd, 0) : MAP_FAILED;
  ::close(fd);
  if (map == MAP_FAILED) { set_create_error("mmap failed"); return nullptr; }
  ParsedFile P;
  std::string perr;
  const bool ok = parse_file(static_cast<const uint8_t*>(map), size, P, perr);
  if (!ok) { munmap(map, size); set_create_error(perr); return nullptr; }
  Engine* E = new Engine();
  E->device = device;
  E->max_batch = max_batch;
  E->max_seq = max_seq;
  E->tp_rank = tp_rank;
  E->tp_world = tp_world;
  bool good;
  {
    DeviceGuard dg(device);
    good = init_device(E, static_cast<const uint8_t*>(map), P);
    if (good && tp_world > 1) good = init_tp(E, *tp_id);
  }
  munmap(map, size);
  if (!good) {
    set_create_error(E->err);
    destroy(E);
    return nullptr;
  }
  return E;
}

// =============================================================================================
// 2-way tensor-parallel batch-1 variant.  Each of the two ranks (one process and one GPU each)
// holds half of every layer: q heads [16r, 16r+16) and kv heads [4r, 4r+4) (rows of Wq, Wk, Wv),
// the matching 1024 columns of W_o, ffn rows [4096r, 4096r+4096) of W_gate / W_up and those
// columns of W_down, and vocabulary rows [64128r, 64128r+64128) of the lm_head.  Per layer the
// o-proj and down partial sums are added across the ranks with one NCCL all-reduce each (rank 0
// adds the residual, rank 1 contributes its partial from zero), and the greedy id is the better
// of the two ranks' candidates (all-gather of (value, index); the lower index wins ties).  The
// step runs the per-phase kernels and is captured into a CUDA graph with the NCCL calls.
// NCCL is loaded at run time, so the engine library has no link-time NCCL dependency.
// =============================================================================================
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

static const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // an NCCL already loaded into the process (e.g. by PyTorch) is found first by its soname
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
             api.error_string;
  });
  return api;
}

#define LE_NCCL(expr)                                                        \
  do {                                                                       \
    ncclResult_t r_ = (expr);                                                \
    if (r_ != ncclSuccess) {                                                 \
      E->err = std::string(#expr) + ": " + nccl().error_string(r_);          \
      return false;                                                          \
    }                                                                        \
  } while (0)

// This rank's greedy candidate with its global index, as (value bits, index).
__global__ void k_tp_candidate(const ArgmaxPart* __restrict__ part, int nparts, int offset, int32_t* __restrict__ out) {
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
    out[0] = __float_as_int(bv);
    out[1] = bi == kNoIndex ? kNoIndex : bi + offset;
  }
}

// The greedy id over all ranks' candidates (the reference's rule: first index among the
// maxima, 0 when none exceeds -1e30); with `advance` the step parameters move on as in
// k_argmax_finish.
__global__ void k_tp_pick(const int32_t* __restrict__ cand, int world, int32_t* __restrict__ result,
                          StepParams* __restrict__ prm, int32_t* __restrict__ token_log, int advance) {
  if (threadIdx.x != 0) return;
  float bv = -1e30f;
  int bi = kNoIndex;
  for (int r = 0; r < world; ++r) argmax_merge(bv, bi, __int_as_float(cand[2 * r]), cand[2 * r + 1]);
  const int id = bi == kNoIndex ? 0 : bi;
  *result = id;
  if (advance) {
    token_log[prm->step] = id;
    prm->step += 1;
    prm->token = id;
    prm->pos += 1;
  }
}

// Captures one tensor-parallel token step (mode 0: no logits, 1: logits gathered on both ranks,
// 2: greedy + advance without gathering the logits).
static bool capture_tp(Engine* E, int mode, cudaGraphExec_t* out) {
  const NcclApi& nc = nccl();
  const int dim = (int)E->dim, ffn = (int)E->ffn, kvh = (int)E->kv_dim / 2;
  const int nq = (int)E->heads / 2, nkv = (int)E->kv_heads / 2;
  const size_t layer_stride = (size_t)E->max_seq * kvh;
  cudaStream_t s = E->stream;
  cudaGraph_t g = nullptr;
  LE_CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  k_embed<<<1, kThreads, 0, s>>>(E->lm_head, E->d_params, nullptr, E->x);
  for (uint32_t l = 0; l < E->layers; ++l) {
    const DevLayer& T = E->tpl[l];
    const int qkv_rows = T.q.N + T.k.N + T.v.N;
    k_qkv<2><<<(qkv_rows / 2 + kWarps - 1) / kWarps, kThreads, gemv_smem(dim), s>>>(E->x, T.in_norm, T.q, T.k, T.v,
                                                                                   E->tp_qkv);
    const size_t att_smem = (size_t)(64 * 3 + 32 + 256 + E->max_seq) * 4;
    k_attention<<<nq, kThreads, att_smem, s>>>(E->tp_qkv, E->tp_kc + l * layer_stride, E->tp_vc + l * layer_stride,
                                               E->rope_cos, E->rope_sin, E->d_params, nq, nkv, E->tp_attn);
    if (E->tp_rank != 0) cudaMemsetAsync(E->x, 0, (size_t)dim * 4, s);
    k_proj_residual<1, 2><<<(dim + kWarps - 1) / kWarps, kThreads, gemv_smem(dim), s>>>(E->tp_attn, T.o, E->x);
    nc.all_reduce(E->x, E->x, (size_t)dim, ncclFloat, ncclSum, E->tp_comm, s);
    k_gateup<2><<<(T.g.N / 2 + kWarps - 1) / kWarps, kThreads, gemv_smem(dim), s>>>(E->x, T.post_norm, T.g, T.u,
                                                                                   E->tp_act);
    if (E->tp_rank != 0) cudaMemsetAsync(E->x, 0, (size_t)dim * 4, s);
    k_proj_residual<1, 8><<<(dim + kWarps - 1) / kWarps, kThreads, gemv_smem(ffn), s>>>(E->tp_act, T.d, E->x);
    nc.all_reduce(E->x, E->x, (size_t)dim, ncclFloat, ncclSum, E->tp_comm, s);
  }
  if (mode != 0) {
    const int half = E->tp_lm.N;
    float* mine = E->logits + (size_t)E->tp_rank * half;
    k_lmhead<2><<<E->lm_grid, kThreads, gemv_smem(dim), s>>>(E->x, E->final_norm, E->tp_lm, mine, E->tp_part);
    k_tp_candidate<<<1, 1024, 0, s>>>(E->tp_part, E->lm_grid, E->tp_rank * half, E->tp_cand + 2 * E->tp_rank);
    nc.all_gather(E->tp_cand + 2 * E->tp_rank, E->tp_cand, 2, ncclInt32, E->tp_comm, s);
    if (mode == 1) nc.all_gather(mine, E->logits, (size_t)half, ncclFloat, E->tp_comm, s);
    k_tp_pick<<<1, 32, 0, s>>>(E->tp_cand, E->tp_world, E->am_result, E->d_params, E->token_log, mode == 2 ? 1 : 0);
  }
  cudaError_t ce = cudaStreamEndCapture(s, &g);
  if (ce != cudaSuccess) { E->err = std::string("tp capture: ") + cudaGetErrorString(ce); return false; }
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) { E->err = std::string("tp instantiate: ") + cudaGetErrorString(ce); return false; }
  return true;
}

static bool init_tp(Engine* E, const ncclUniqueId& id) {
  const NcclApi& nc = nccl();
  if (!nc.ok) { E->err = "tensor parallel: NCCL (libnccl.so.2) could not be loaded"; return false; }
  const int r = E->tp_rank, W = E->tp_world;
  if (W != 2 || E->heads % 4 || E->kv_heads % 2 || E->dim % 256 || E->ffn % 256 || E->vocab % 32 ||
      (E->heads / 2) % (E->kv_heads / 2)) {
    E->err = "tensor parallel: needs 2 ranks and a geometry that halves on 128-blocks";
    return false;
  }
  const int dim = (int)E->dim, ffn = (int)E->ffn, kv = (int)E->kv_dim;
  // row slices are views of the uploaded matrices
  auto rows = [](const QMat& M, int n0, int n) {
    QMat q = M;
    q.nib = M.nib + (size_t)n0 * (M.K / 2);
    q.step = M.step + (size_t)n0 * (M.K / 128);
    q.mn = M.mn + (size_t)n0 * (M.K / 128);
    q.N = n;
    return q;
  };
  // column halves are copied into a contiguous matrix (2-D copies of the nibble and scale rows)
  const size_t o_half = (size_t)dim * (dim / 2), d_half = (size_t)dim * (ffn / 2);  // weights per half
  auto mat_bytes = [](size_t w) { return align_up(w / 2, 256) + 2 * align_up(w / 128 * 2, 256); };
  const size_t tp_bytes = E->layers * (mat_bytes(o_half) + mat_bytes(d_half));
  LE_CK(cudaMalloc(&E->tp_arena, tp_bytes));
  size_t off = 0;
  auto cols = [&](const QMat& M, int k0, int k) -> QMat {
    QMat q;
    q.N = M.N;
    q.K = k;
    uint8_t* nib = E->tp_arena + off;
    off += align_up((size_t)M.N * k / 2, 256);
    uint16_t* st = reinterpret_cast<uint16_t*>(E->tp_arena + off);
    off += align_up((size_t)M.N * (k / 128) * 2, 256);
    uint16_t* mn = reinterpret_cast<uint16_t*>(E->tp_arena + off);
    off += align_up((size_t)M.N * (k / 128) * 2, 256);
    cudaMemcpy2DAsync(nib, k / 2, M.nib + k0 / 2, M.K / 2, k / 2, M.N, cudaMemcpyDeviceToDevice, E->stream);
    cudaMemcpy2DAsync(st, (k / 128) * 2, M.step + k0 / 128, (M.K / 128) * 2, (k / 128) * 2, M.N,
                      cudaMemcpyDeviceToDevice, E->stream);
    cudaMemcpy2DAsync(mn, (k / 128) * 2, M.mn + k0 / 128, (M.K / 128) * 2, (k / 128) * 2, M.N,
                      cudaMemcpyDeviceToDevice, E->stream);
    q.nib = nib;
    q.step = st;
    q.mn = mn;
    return q;
  };
  E->tpl.resize(E->layers);
  for (uint32_t l = 0; l < E->layers; ++l) {
    const DevLayer& D = E->L[l];
    DevLayer& T = E->tpl[l];
    T.in_norm = D.in_norm;
    T.post_norm = D.post_norm;
    T.q = rows(D.q, r * dim / 2, dim / 2);
    T.k = rows(D.k, r * kv / 2, kv / 2);
    T.v = rows(D.v, r * kv / 2, kv / 2);
    T.o = cols(D.o, r * dim / 2, dim / 2);
    T.g = rows(D.g, r * ffn / 2, ffn / 2);
    T.u = rows(D.u, r * ffn / 2, ffn / 2);
    T.d = cols(D.d, r * ffn / 2, ffn / 2);
  }
  LE_CK(cudaGetLastError());
  E->tp_lm = rows(E->lm_head, r * (int)E->vocab / 2, (int)E->vocab / 2);
  const size_t kv_elems = (size_t)E->layers * E->max_seq * (kv / 2);
  LE_CK(cudaMalloc(&E->tp_kc, kv_elems * 4));
  LE_CK(cudaMalloc(&E->tp_vc, kv_elems * 4));
  LE_CK(cudaMemsetAsync(E->tp_kc, 0, kv_elems * 4, E->stream));
  LE_CK(cudaMemsetAsync(E->tp_vc, 0, kv_elems * 4, E->stream));
  LE_CK(cudaMalloc(&E->tp_qkv, (size_t)(dim + 2 * kv) / 2 * 4));
  LE_CK(cudaMalloc(&E->tp_attn, (size_t)dim / 2 * 4));
  LE_CK(cudaMalloc(&E->tp_act, (size_t)ffn / 2 * 4));
  LE_CK(cudaMalloc(&E->tp_part, (size_t)E->lm_grid * sizeof(ArgmaxPart)));
  LE_CK(cudaMalloc(&E->tp_cand, (size_t)W * 2 * 4));
  LE_CK(cudaStreamSynchronize(E->stream));
  LE_NCCL(nc.comm_init_rank(&E->tp_comm, W, id, r));
  for (int m = 0; m < 3; ++m)
    if (!capture_tp(E, m, &E->tp_g[m])) return false;
  return true;
}

static void destroy_tp(Engine* E) {
  for (auto& g : E->tp_g)
    if (g) { cudaGraphExecDestroy(g); g = nullptr; }  // graphs holding NCCL calls go first
  if (E->tp_comm) { nccl().comm_destroy(E->tp_comm); E->tp_comm = nullptr; }
  void* p[] = {E->tp_arena, E->tp_kc, E->tp_vc, E->tp_qkv, E->tp_attn, E->tp_act, E->tp_part, E->tp_cand};
  for (void* q : p) if (q) cudaFree(q);
  E->tp_arena = nullptr;
  E->tp_kc = E->tp_vc = E->tp_qkv = E->tp_attn = E->tp_act = nullptr;
  E->tp_part = nullptr;
  E->tp_cand = nullptr;
}

static bool queue_params(Engine* E, int32_t token, int32_t pos) {
  const int slot = E->ring_pos;
  E->ring_pos = (E->ring_pos + 1) % kRing;
  if (E->ring_used[slot]) LE_CK(cudaEventSynchronize(E->ring_ev[slot]));
  E->h_ring[slot] = StepParams{token, pos, 0, 0};
  E->last_pos = pos;
  LE_CK(cudaMemcpyAsync(E->d_params, &E->h_ring[slot], sizeof(StepParams), cudaMemcpyHostToDevice, E->stream));
  LE_CK(cudaEventRecord(E->ring_ev[slot], E->stream));
  E->ring_used[slot] = true;
  return true;
}

static bool forward_token(Engine* E, int32_t token, size_t pos, bool logits) {
  if (pos >= (size_t)E->max_seq) return true;  // silent no-op, src/llama_engine.cpp:936
  if (token < 0 || token >= (int32_t)E->vocab) token = 0;  // :937
  if (E->persist) {
    E->last_pos = (int32_t)pos;
    if (!launch_persistent(E, 1, logits, token, (int32_t)pos)) return false;
  } else {
    if (!queue_params(E, token, (int32_t)pos)) return false;
    if (E->tp_world > 1) {
      LE_CK(cudaGraphLaunch(E->tp_g[logits ? 1 : 0], E->stream));
    } else {
      LE_CK(cudaGraphLaunch(E->g_fwd[logits ? 1 : 0], E->stream));
    }
  }
  if (logits) {
    E->logits_on_host_fresh = false;
    set_argmax(E, true, E->persist);
    E->have_logits = true;
  }
  return true;
}

// Waits for the newest persistent launch through the mapped completion words (the kernel's last
// CTA writes them as it finishes) instead of a device-to-host copy and a stream wait.  Returns
// false when that cannot be used (the stream drained without the words: the slow path reads the
// result instead) and sets *failed on a CUDA error.
static bool wait_done_words(Engine* E, bool* failed) {
  volatile uint32_t* hd = E->h_done;
  const uint32_t want = E->persist_seq;
  for (uint32_t i = 1;; ++i) {
    if (hd[3] == want) break;
    if ((i & 255) == 0) {  // now and then: has the stream drained, or failed?
      const cudaError_t q = cudaStreamQuery(E->stream);
      if (q == cudaSuccess) {
        if (hd[3] == want) break;
        return false;
      }
      if (q != cudaErrorNotReady) {
        E->err = cudaGetErrorString(q);
        *failed = true;
        return false;
      }
    }
  }
  std::atomic_thread_fence(std::memory_order_acquire);  // the words before seq
  return true;
}

static bool greedy(Engine* E, int32_t* out) {
  if (E->argmax_valid && E->argmax_persist && E->h_done && E->persist_seq_logits == E->persist_seq &&
      !(E->tc && E->tc_dirty)) {
    bool failed = false;
    if (wait_done_words(E, &failed)) {
      E->h_err[0] = E->h_done[0];
      E->h_err[1] = E->h_done[1];
      if (!check_status(E)) return false;
      *out = (int32_t)E->h_done[2];
      return true;
    }
    if (failed) return false;
  }
  if (!E->argmax_valid) {
    const int parts = std::min<int>(E->num_sms * 2, (E->vocab + kThreads - 1) / kThreads);
    k_argmax_rows<<<parts, kThreads, 0, E->stream>>>(E->logits, E->vocab, E->part);
    k_argmax_finish<<<1, 1024, 0, E->stream>>>(E->part, parts, E->am_result, E->d_params, E->token_log, 0);
    LE_CK(cudaGetLastError());
    set_argmax(E, true);
  }
  if (E->persist && !(E->tc && E->tc_dirty)) {
    // one copy for the persistent kernel's error words and am_result[0], which follows PCtrl
    constexpr size_t off = offsetof(PCtrl, error), bytes = sizeof(PCtrl) + 4 - off;
    static_assert(bytes % 4 == 0 && offsetof(PCtrl, err_where) == off + 4, "PCtrl layout");
    LE_CK(cudaMemcpyAsync(E->h_small, E->ctrl_block + off, bytes, cudaMemcpyDeviceToHost, E->stream));
    LE_CK(cudaStreamSynchronize(E->stream));
    E->h_err[0] = (uint32_t)E->h_small[0];
    E->h_err[1] = (uint32_t)E->h_small[1];
    if (!check_status(E)) return false;
    *out = E->h_small[bytes / 4 - 1];
    return true;
  }
  LE_CK(cudaMemcpyAsync(E->h_small, E->am_result, 4, cudaMemcpyDeviceToHost, E->stream));
  if (!enqueue_status(E)) return false;
  LE_CK(cudaStreamSynchronize(E->stream));  // one wait for the id and the error words
  if (!check_status(E)) return false;
  *out = E->h_small[0];
  return true;
}

static bool sync_logits(Engine* E) {
  if (!E->logits_on_host_fresh) {
    LE_CK(cudaMemcpyAsync(E->h_logits, E->logits, (size_t)E->vocab * 4, cudaMemcpyDeviceToHost, E->stream));
    LE_CK(cudaStreamSynchronize(E->stream));
    if (!persistent_ok(E)) return false;
    E->logits_on_host_fresh = true;
  }
  return true;
}

// Temperature / top-p sampling.  The probabilities are formed on the device; the candidate walk of
// sample_top_p (src/llama_engine.cpp:808-838) runs over the host mirror, with libc rand().
// The draw over the candidates (src/llama_engine.cpp:824-838): the shortest prefix whose mass
// reaches top_p, a libc rand() point in it, the first candidate whose running mass reaches it.
static int32_t draw_top_p(const int32_t* ids, const float* vals, size_t k, float top_p) {
  float cum = 0.0f;
  size_t last = 0;
  for (size_t i = 0; i < k; ++i) { cum += vals[i]; last = i; if (cum >= top_p) break; }
  const float r = (static_cast<float>(rand()) / static_cast<float>(RAND_MAX)) * cum;
  float run = 0.0f;
  for (size_t i = 0; i <= last; ++i) { run += vals[i]; if (run >= r) return ids[i]; }
  return ids[0];
}

static int32_t sample_top_p_host(float* p, size_t vocab, float top_p) {
  const size_t k = std::min<size_t>(64, vocab);
  int32_t ids[64];
  float vals[64];
  for (size_t i = 0; i < k; ++i) { ids[i] = (int32_t)i; vals[i] = p[i]; }
  for (size_t i = k; i < vocab; ++i) {
    const float v = p[i];
    if (v > vals[k - 1]) {
      size_t q = k - 1;
      while (q > 0 && v > vals[q - 1]) { vals[q] = vals[q - 1]; ids[q] = ids[q - 1]; --q; }
      vals[q] = v; ids[q] = (int32_t)i;
    }
  }
  return draw_top_p(ids, vals, k, top_p);
}

}  // namespace le

#include "sampler_kernels.cuh"

using namespace le;

// =============================================================================================
// C ABI, Part 1 (reference entry points)
// =============================================================================================

static Engine* H(llama_engine_t e) { return static_cast<Engine*>(e); }

static int default_device() {
  const char* d = getenv("LLAMA_ENGINE_DEVICE");
  return d ? atoi(d) : 0;
}

LE_API llama_engine_t llama_engine_create(const char* model_path) {
  return create(model_path, default_device(), 1, LE_MAX_SEQ_LEN);
}

LE_API void llama_engine_free(llama_engine_t engine) { destroy(H(engine)); }

LE_API void llama_engine_reset(llama_engine_t engine) { (void)engine; }

LE_API int32_t llama_engine_get_num_layers(llama_engine_t e) { return e ? (int32_t)H(e)->layers : 0; }
LE_API int32_t llama_engine_get_dim(llama_engine_t e) { return e ? (int32_t)H(e)->dim : 0; }
LE_API int32_t llama_engine_get_ffn_dim(llama_engine_t e) { return e ? (int32_t)H(e)->ffn : 0; }
LE_API int32_t llama_engine_get_vocab_size(llama_engine_t e) { return e ? (int32_t)H(e)->vocab : 0; }
LE_API int32_t llama_engine_get_num_heads(llama_engine_t e) { return e ? (int32_t)H(e)->heads : 0; }
LE_API int32_t llama_engine_get_num_kv_heads(llama_engine_t e) { return e ? (int32_t)H(e)->kv_heads : 0; }
LE_API int32_t llama_engine_get_head_dim(llama_engine_t e) { return e ? (int32_t)LE_HEAD_DIM : 0; }
LE_API int32_t llama_engine_get_max_seq_len(llama_engine_t e) { (void)e; return LE_MAX_SEQ_LEN; }

LE_API int llama_engine_forward_token(llama_engine_t engine, int32_t token_id, size_t pos, int compute_logits) {
  if (!engine) return -1;
  Engine* E = H(engine);
  DeviceGuard dg(E->device);
  return forward_token(E, token_id, pos, compute_logits != 0) ? 0 : -1;
}

LE_API int llama_engine_prefill(llama_engine_t engine, const int32_t* token_ids, size_t count, size_t start_pos,
                                int compute_last_logits) {
  if (!engine || !token_ids) return -1;
  Engine* E = H(engine);
  DeviceGuard dg(E->device);
  // positions at or past max_seq_len are silent no-ops (src/llama_engine.cpp:936)
  if (start_pos >= (size_t)E->max_seq) return 0;
  const size_t n = std::min(count, (size_t)E->max_seq - start_pos);
  const bool last = compute_last_logits != 0 && n == count;
  if (E->tc && n >= 2) {
    if (!tc_prefill(E, token_ids, n, start_pos, last)) return -1;
    if (last) {
      E->logits_on_host_fresh = false;
      set_argmax(E, true);
      E->have_logits = true;
    }
    return 0;
  }
  for (size_t i = 0; i < n; ++i) {
    if (!forward_token(E, token_ids[i], start_pos + i, last && i + 1 == n)) return -1;
  }
  return 0;
}

LE_API int32_t llama_engine_sample(llama_engine_t engine, float temperature, float top_p) {
  if (!engine) return 0;
  Engine* E = H(engine);
  DeviceGuard dg(E->device);
  int32_t id = 0;
  if (temperature <= 0.01f) {
    if (!greedy(E, &id)) return 0;
    return id;
  }
  if (!softmax_in_place(E, temperature)) return 0;
  if (E->vocab < 64) {
    if (!sync_logits(E)) return 0;
    return sample_top_p_host(E->h_logits, E->vocab, top_p);
  }
  // the 64 candidates on the device; the draw (libc rand(), :824-838) on the host
  int32_t* d_ids = reinterpret_cast<int32_t*>(E->red + 1536);
  float* d_vals = E->red + 1600;
  k_topk64_walk<<<1, 256, 0, E->stream>>>(E->logits, (int)E->vocab, d_ids, d_vals);
  if (cudaGetLastError() != cudaSuccess) return 0;
  if (cudaMemcpyAsync(E->h_small, d_ids, 128 * 4, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess) return 0;
  if (!sync_ok(E)) return 0;
  return draw_top_p(E->h_small, reinterpret_cast<const float*>(E->h_small + 64), 64, top_p);
}

LE_API const float* llama_engine_get_logits(llama_engine_t engine) {
  if (!engine) return nullptr;
  Engine* E = H(engine);
  DeviceGuard dg(E->device);
  if (!sync_logits(E)) return nullptr;
  return E->h_logits;
}

LE_API void llama_engine_dequantize_embedding(llama_engine_t engine, size_t token_id, float* out_x) {
  if (!engine || !out_x) return;
  Engine* E = H(engine);
  if (token_id >= E->vocab) return;
  DeviceGuard dg(E->device);
  int32_t* tok = E->d_misc;
  if (cudaStreamSynchronize(E->stream) != cudaSuccess) return;  // h_small may be in use by a copy
  E->h_small[0] = (int32_t)token_id;
  if (cudaMemcpyAsync(tok, E->h_small, 4, cudaMemcpyHostToDevice, E->stream) != cudaSuccess) return;
  k_embed<<<1, kThreads, 0, E->stream>>>(E->lm_head, E->d_params, tok, E->emb);
  if (cudaMemcpyAsync(out_x, E->emb, (size_t)E->dim * 4, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess) return;
  cudaStreamSynchronize(E->stream);
}

// =============================================================================================
// C ABI, Part 2 (extensions)
// =============================================================================================

LE_API llama_engine_t llama_engine_create_ex(const char* model_path, int device, int max_batch, int max_seq_len) {
  return create(model_path, device, max_batch, max_seq_len);
}

LE_API const char* llama_engine_last_error(llama_engine_t engine) {
  if (engine) return H(engine)->err.c_str();
  std::lock_guard<std::mutex> lk(g_err_mu);
  static thread_local std::string copy;
  copy = g_create_error;
  return copy.c_str();
}

LE_API int llama_engine_generate_greedy(llama_engine_t engine, int32_t first_token, size_t start_pos,
                                        int32_t n_steps, int32_t* out_tokens) {
  if (!engine || !out_tokens || n_steps < 0) return -1;
  Engine* E = H(engine);
  if (n_steps == 0) return 0;
  if (start_pos + (size_t)n_steps > (size_t)E->max_seq) { E->err = "generate_greedy: positions exceed max_seq_len"; return -1; }
  DeviceGuard dg(E->device);
  if (first_token < 0 || first_token >= (int32_t)E->vocab) first_token = 0;
  if (!queue_params(E, first_token, (int32_t)start_pos)) return -1;
  E->last_pos = (int32_t)(start_pos + n_steps - 1);
  if (E->tp_world > 1) {
    for (int32_t i = 0; i < n_steps; ++i)
      if (cudaGraphLaunch(E->tp_g[2], E->stream) != cudaSuccess) { E->err = "graph launch failed"; return -1; }
  } else if (E->persist) {
    if (!launch_persistent(E, n_steps, true, first_token, (int32_t)start_pos)) return -1;
  } else {
    for (int32_t i = 0; i < n_steps; ++i)
      if (cudaGraphLaunch(E->g_gen, E->stream) != cudaSuccess) { E->err = "graph launch failed"; return -1; }
  }
  if (cudaMemcpyAsync(out_tokens, E->token_log, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess)
    return -1;
  cudaError_t ce = cudaStreamSynchronize(E->stream);
  if (ce != cudaSuccess) { E->err = cudaGetErrorString(ce); return -1; }
  if (!persistent_ok(E)) return -1;
  E->logits_on_host_fresh = false;
  set_argmax(E, true);
  E->have_logits = true;
  return 0;
}

LE_API int llama_engine_forward_batch(llama_engine_t engine, const int32_t* tokens, const int32_t* positions,
                                      const int32_t* slots, int n, int compute_logits) {
  if (!engine || !tokens || !positions || !slots || n < 1) return -1;
  Engine* E = H(engine);
  // the batched path takes up to tc_T rows (several positions of a slot may share a call); rows
  // with logits land in the max_batch logits rows
  const int max_rows = E->tc ? std::max(E->max_batch, E->tc_T) : E->max_batch;
  if (n > max_rows || (compute_logits && n > E->max_batch)) {
    E->err = "forward_batch: n exceeds the row capacity";
    return -1;
  }
  for (int i = 0; i < n; ++i) {
    if (slots[i] < 0 || slots[i] >= E->max_batch) { E->err = "forward_batch: slot out of range"; return -1; }
    if (positions[i] < 0 || positions[i] >= E->max_seq) { E->err = "forward_batch: position out of range"; return -1; }
  }
  {  // two rows for the same (slot, position) would both append its k / v: rejected
    std::vector<std::pair<int32_t, int32_t>> sp(n);
    for (int i = 0; i < n; ++i) sp[i] = {slots[i], positions[i]};
    std::sort(sp.begin(), sp.end());
    if (std::adjacent_find(sp.begin(), sp.end()) != sp.end()) {
      E->err = "forward_batch: two rows for the same (slot, position)";
      return -1;
    }
  }
  DeviceGuard dg(E->device);
  if (E->tc) {
    if (!tc_upload_rows(E, tokens, positions, slots, n)) return -1;
    // stream-ordered: a device error (the GEMM's bounded waits) is reported by the next call
    // that synchronises (argmax_batch, get_logits_batch, get_logits, sample)
    // RoPE / KV append inside attention only when no slot repeats (a row may read the k / v
    // that an earlier row of the same call appends)
    std::vector<uint8_t> seen(E->max_batch, 0);
    bool distinct = true;
    for (int i = 0; i < n && distinct; ++i) distinct = !seen[slots[i]]++;
    if (!tc_step_graph(E, n, compute_logits ? n : 0, *std::max_element(positions, positions + n), distinct))
      return -1;
    E->logits_on_host_fresh = false;
    if (compute_logits) { set_argmax(E, true); E->have_logits = true; }
    return 0;
  }
  std::vector<StepParams> hp(n);
  for (int i = 0; i < n; ++i) {
    int32_t t = tokens[i];
    if (t < 0 || t >= (int32_t)E->vocab) t = 0;
    hp[i] = StepParams{t, positions[i], 0, 0};
  }
  if (cudaMemcpyAsync(E->d_params, hp.data(), n * sizeof(StepParams), cudaMemcpyHostToDevice, E->stream) != cudaSuccess)
    return -1;
  for (int i = 0; i < n; ++i) enqueue_token(E, row_buffers(E, i, slots[i], compute_logits != 0, 0), E->stream);
  cudaError_t ce = cudaStreamSynchronize(E->stream);  // hp goes out of scope
  if (ce != cudaSuccess) { E->err = cudaGetErrorString(ce); return -1; }
  E->logits_on_host_fresh = false;
  if (compute_logits) { set_argmax(E, true); E->have_logits = true; }
  return 0;
}

LE_API int llama_engine_trace(llama_engine_t engine, int enable, unsigned long long* out, int max_entries) {
  if (!engine) return -1;
  Engine* E = H(engine);
  if (!E->persist) return -1;
  DeviceGuard dg(E->device);
  const size_t n = (size_t)E->p_grid * kTraceCap * 2;
  if (enable == 1) {
    if (!E->d_trace && cudaMalloc(&E->d_trace, n * 8) != cudaSuccess) return -1;
    if (cudaMemsetAsync(E->d_trace, 0, n * 8, E->stream) != cudaSuccess) return -1;
    E->pargs.trace = E->d_trace;
    return 0;
  }
  if (enable == 0) {
    E->pargs.trace = nullptr;
    return 0;
  }
  // enable == 2: copy out (grid * kTraceCap pairs of (globaltimer ns, tag))
  if (!E->d_trace || !out) return -1;
  const size_t m = std::min<size_t>(n, (size_t)std::max(0, max_entries) * 2);
  if (cudaMemcpyAsync(out, E->d_trace, m * 8, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess) return -1;
  if (cudaStreamSynchronize(E->stream) != cudaSuccess) return -1;
  return (int)std::min<size_t>((size_t)E->p_grid * kTraceCap, (size_t)std::max(0, max_entries));
}

LE_API int llama_engine_rope_table(float factor, float low_freq_factor, float high_freq_factor,
                                   int original_max_position, int n_pos, float* cos_out, float* sin_out) {
  if (!cos_out || !sin_out || n_pos < 1 || n_pos > LE_MAX_SEQ_LEN) return -1;
  if (factor > 0.0f && !(high_freq_factor > low_freq_factor && low_freq_factor > 0.0f && original_max_position > 0))
    return -1;
  RopeScaling rs{factor, low_freq_factor, high_freq_factor, original_max_position};
  std::vector<float> cs, sn;
  build_rope_table(rs, n_pos, cs, sn);
  std::memcpy(cos_out, cs.data(), cs.size() * 4);
  std::memcpy(sin_out, sn.data(), sn.size() * 4);
  return 0;
}

LE_API int llama_engine_set_rope_scaling(llama_engine_t engine, float factor, float low_freq_factor,
                                         float high_freq_factor, int original_max_position) {
  if (!engine) return -1;
  Engine* E = H(engine);
  if (factor > 0.0f && !(high_freq_factor > low_freq_factor && low_freq_factor > 0.0f && original_max_position > 0)) {
    E->err = "set_rope_scaling: bad parameters";
    return -1;
  }
  DeviceGuard dg(E->device);
  RopeScaling rs{factor, low_freq_factor, high_freq_factor, original_max_position};
  std::vector<float> cs, sn;
  build_rope_table(rs, LE_MAX_SEQ_LEN, cs, sn);
  // queued steps read the table: replace it only after they are done
  cudaError_t ce = cudaStreamSynchronize(E->stream);
  if (ce == cudaSuccess) ce = cudaMemcpy(E->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemcpy(E->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) { E->err = cudaGetErrorString(ce); return -1; }
  return 0;
}

LE_API int llama_engine_check_schedule(int layers, int dim, int ffn_dim, int vocab_size, int num_heads,
                                       int num_kv_heads, int grid, char* err, int err_len) {
  std::string msg;
  bool ok = layers > 0 && dim == 2048 && ffn_dim % 2048 == 0 && ffn_dim > 0 && ffn_dim <= 8192 && vocab_size > 0 &&
            vocab_size % 16 == 0 && num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
            dim / num_heads == LE_HEAD_DIM && grid > 0 && grid <= 1024;
  if (!ok) msg = "unsupported geometry or grid";
  if (ok) {
    PGeom geo{layers, dim, ffn_dim, vocab_size, num_heads, num_kv_heads};
    PSchedule P;
    ok = build_schedule(geo, grid, P, msg) && check_schedule(geo, grid, P, msg);
  }
  if (err && err_len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)err_len - 1);
    err[err_len - 1] = '\0';
  }
  return ok ? 0 : -1;
}

LE_API int llama_b128_gemm_plan(int num_sms, int tiles, int kb, int img_tiles, int splits_req, int32_t* out) {
  if (!out || num_sms < 1 || num_sms > 4096 || tiles < 1 || kb < 1 || img_tiles < 1 || splits_req > kb) return -1;
  const TcPlan pl = tc_plan(num_sms, tiles, kb, img_tiles, splits_req);
  out[0] = pl.P;
  out[1] = pl.groups;
  out[2] = pl.splits;
  out[3] = pl.kb_split;
  return 0;
}

LE_API int llama_engine_debug_waits(llama_engine_t engine, unsigned long long wait_ns, int expire_code) {
  if (!engine) return -1;
  Engine* E = H(engine);
  DeviceGuard dg(E->device);
  if (cudaStreamSynchronize(E->stream) != cudaSuccess) return -1;
  const unsigned long long ns = wait_ns ? wait_ns : kWaitNs;
  E->pargs.wait_ns = ns;
  E->pargs.expire_where = expire_code;
  // expiring only the attention keeps the default bound on the GEMMs: with programmatic launches
  // the next GEMM may already wait for the stalled attention's output, and its bounded waits
  // would otherwise run out in the same millisecond and race the attention's error code
  E->tc_wait_ns = expire_code == kExpireAttn ? kWaitNs : ns;
  E->attn_wait_ns = ns;
  E->tc_expire = expire_code != 0 && expire_code != kExpireAttn ? 1 : 0;
  E->attn_expire = expire_code == kExpireAttn ? 1 : 0;
  // captured batched steps hold the old GEMM arguments
  for (auto& g : E->tc_graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  E->tc_graphs.clear();
  if (expire_code == 0) {  // clear a recorded timeout so the engine can run again
    if (E->persist && cudaMemsetAsync(&E->d_ctrl->error, 0, 2 * sizeof(uint32_t), E->stream) != cudaSuccess) return -1;
    if (E->tc && cudaMemsetAsync(E->tc_err, 0, sizeof(uint32_t), E->stream) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(E->stream) != cudaSuccess) return -1;
    E->h_err[0] = E->h_err[1] = E->h_err[2] = 0;
    E->tc_dirty = true;
  }
  return 0;
}

LE_API int llama_engine_decode_path(llama_engine_t engine) {
  if (!engine) return -1;
  return H(engine)->tp_world > 1 ? 2 : H(engine)->persist ? 1 : 0;
}

LE_API int llama_engine_tp_unique_id(void* out_id, int len) {
  if (!out_id || len < (int)sizeof(ncclUniqueId)) return -1;
  const NcclApi& nc = nccl();
  if (!nc.ok) return -1;
  ncclUniqueId id;
  if (nc.get_unique_id(&id) != ncclSuccess) return -1;
  std::memcpy(out_id, &id, sizeof(id));
  return 0;
}

LE_API llama_engine_t llama_engine_create_tp(const char* model_path, int device, int rank, int world,
                                             const void* unique_id, int max_seq_len) {
  if (!unique_id || world != 2 || rank < 0 || rank >= world) {
    set_create_error("create_tp: needs world = 2, 0 <= rank < world and the rank-0 unique id");
    return nullptr;
  }
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  return create(model_path, device, 1, max_seq_len, rank, world, &id);
}

LE_API int llama_engine_batch_path(llama_engine_t engine) {
  if (!engine) return -1;
  return H(engine)->tc ? 1 : 0;
}

LE_API void* llama_engine_get_stream(llama_engine_t engine) { return engine ? (void*)H(engine)->stream : nullptr; }

LE_API int llama_engine_profile_phase(llama_engine_t engine, const char* phase, int iters, float* avg_ms) {
  if (!engine || !phase || iters < 1 || !avg_ms) return -1;
  Engine* E = H(engine);
  static const char* names[] = {"qkv", "attn", "oproj", "gateup", "down", "lmhead"};
  int ph = -1;
  for (int i = 0; i < 6; ++i)
    if (std::strcmp(phase, names[i]) == 0) ph = i;
  const bool step = std::strcmp(phase, "step") == 0;
  if (ph < 0 && !step) { E->err = "profile_phase: unknown phase"; return -1; }
  DeviceGuard dg(E->device);
  cudaEvent_t a, b;
  if (cudaEventCreate(&a) != cudaSuccess) return -1;
  if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return -1; }
  TokenBuffers B = row_buffers(E, 0, 0, true, 0);
  // device params may have been advanced past the cache by a generation: re-queue a valid one
  if (!queue_params(E, 0, std::min<int32_t>(E->last_pos, E->max_seq - 1))) {
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return -1;
  }
  cudaEventRecord(a, E->stream);
  for (int i = 0; i < iters; ++i) {
    if (step) {
      if (E->persist) launch_persistent(E, 1, true, 0, std::min<int32_t>(E->last_pos, E->max_seq - 1));
      else cudaGraphLaunch(E->g_fwd[1], E->stream);
    }
    else enqueue_phase(E, B, ph, (uint32_t)(i % E->layers), E->stream);
  }
  cudaEventRecord(b, E->stream);
  cudaError_t ce = cudaEventSynchronize(b);
  float ms = 0.0f;
  if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (ce != cudaSuccess) { E->err = cudaGetErrorString(ce); return -1; }
  *avg_ms = ms / (float)iters;
  E->logits_on_host_fresh = false;
  set_argmax(E, false);
  return 0;
}

LE_API int llama_engine_argmax_batch(llama_engine_t engine, int32_t* out_tokens, int n) {
  if (!engine || !out_tokens || n < 1) return -1;
  Engine* E = H(engine);
  if (n > E->max_batch) return -1;
  DeviceGuard dg(E->device);
  if (cudaMemcpyAsync(out_tokens, E->am_result, (size_t)n * 4, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess) return -1;
  return sync_ok(E) ? 0 : -1;  // reports a device error of the step
}

LE_API const float* llama_engine_get_logits_batch(llama_engine_t engine, int row) {
  if (!engine) return nullptr;
  Engine* E = H(engine);
  if (row < 0 || row >= E->max_batch) return nullptr;
  DeviceGuard dg(E->device);
  float* h = E->h_logits + (size_t)row * E->vocab;
  if (cudaMemcpyAsync(h, E->logits + (size_t)row * E->vocab, (size_t)E->vocab * 4, cudaMemcpyDeviceToHost,
                      E->stream) != cudaSuccess)
    return nullptr;
  if (!sync_ok(E)) return nullptr;  // reports a device error of the step
  if (row == 0) E->logits_on_host_fresh = true;
  return h;
}

// ---------------------------------------------------------------------------------------------
// Token scoring for log-likelihood consumers (the lm-eval adapter pattern,
// tests/lm_eval_adapter.py:111-229): one pass over a token run on slot 0, log-probabilities of
// each next token computed on the device.
// ---------------------------------------------------------------------------------------------
static bool score_alloc(Engine* E) {
  if (E->sc_logits) return true;
  LE_CK(cudaMalloc(&E->sc_logits, (size_t)kScoreRows * E->vocab * 4));
  LE_CK(cudaMalloc(&E->sc_target, kScoreRows * 4));
  LE_CK(cudaMalloc(&E->sc_lp, kScoreRows * 4));
  LE_CK(cudaMalloc(&E->sc_greedy, kScoreRows * 4));
  return true;
}

LE_API int llama_engine_score_tokens(llama_engine_t engine, const int32_t* tokens, size_t n, size_t start_pos,
                                     float* out_logprobs, int32_t* out_greedy) {
  if (!engine || !tokens || !out_logprobs || n < 2) return -1;
  Engine* E = H(engine);
  if (start_pos + n > (size_t)E->max_seq) { E->err = "score_tokens: positions exceed max_seq_len"; return -1; }
  DeviceGuard dg(E->device);
  if (!score_alloc(E)) return -1;
  std::vector<int32_t> ids(n), pos(n), slot(n, 0), tgt(kScoreRows);
  for (size_t i = 0; i < n; ++i) {
    ids[i] = (tokens[i] < 0 || tokens[i] >= (int32_t)E->vocab) ? 0 : tokens[i];
    pos[i] = (int32_t)(start_pos + i);
  }
  const int chunk = E->tc ? std::min(E->tc_T, kScoreRows) : 1;
  for (size_t c0 = 0; c0 < n; c0 += (size_t)chunk) {
    const int m = (int)std::min<size_t>((size_t)chunk, n - c0);
    if (E->tc) {
      if (!tc_upload_rows(E, ids.data() + c0, pos.data() + c0, slot.data(), m)) return -1;
      if (!tc_step(E, m, 0, m, pos[c0 + m - 1], pos[c0], E->sc_logits)) return -1;
    } else {
      if (!forward_token(E, ids[c0], (size_t)pos[c0], true)) return -1;
      if (cudaMemcpyAsync(E->sc_logits, E->logits, (size_t)E->vocab * 4, cudaMemcpyDeviceToDevice, E->stream) !=
          cudaSuccess)
        return -1;
    }
    // row i scores token c0 + i + 1 (the run's last token has no successor)
    for (int i = 0; i < m; ++i) tgt[i] = c0 + i + 1 < n ? ids[c0 + i + 1] : -1;
    if (cudaMemcpyAsync(E->sc_target, tgt.data(), (size_t)m * 4, cudaMemcpyHostToDevice, E->stream) != cudaSuccess)
      return -1;
    k_logprob_rows<<<m, 1024, 0, E->stream>>>(E->sc_logits, (int)E->vocab, E->vocab, E->sc_target, E->sc_lp,
                                                E->sc_greedy);
    const int k = (int)std::min<size_t>((size_t)m, n - 1 - c0);
    if (k > 0) {
      if (cudaMemcpyAsync(out_logprobs + c0, E->sc_lp, (size_t)k * 4, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess)
        return -1;
      if (out_greedy &&
          cudaMemcpyAsync(out_greedy + c0, E->sc_greedy, (size_t)k * 4, cudaMemcpyDeviceToHost, E->stream) != cudaSuccess)
        return -1;
    }
    if (c0 + m == n) {  // the last token's logits become the current logits (as after prefill)
      if (cudaMemcpyAsync(E->logits, E->sc_logits + (size_t)(m - 1) * E->vocab, (size_t)E->vocab * 4,
                          cudaMemcpyDeviceToDevice, E->stream) != cudaSuccess)
        return -1;
    }
    // tgt and the host outputs are reused / read by the caller: finish the chunk
    cudaError_t ce = cudaStreamSynchronize(E->stream);
    if (ce != cudaSuccess) { E->err = cudaGetErrorString(ce); return -1; }
  }
  if (!persistent_ok(E)) return -1;
  E->logits_on_host_fresh = false;
  set_argmax(E, false);
  E->have_logits = true;
  return 0;
}

// ---------------------------------------------------------------------------------------------
// Isolated GEMV
// ---------------------------------------------------------------------------------------------
template <int MX, int R, int CPL>
static int launch_gemv(const QMat& W, const float* x, float* y, cudaStream_t s, int num_sms) {
  const size_t smem = (size_t)MX * (W.K + W.K / 128) * 4;
  if (smem > 200 * 1024) return -1;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(k_gemv<MX, R, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return -1;
  const int groups = W.N / R;
  const int grid = std::min<int>((groups + kWarps - 1) / kWarps, num_sms * 8);
  k_gemv<MX, R, CPL><<<grid, kThreads, smem, s>>>(x, W, y);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <int R, int CPL>
static int launch_gemv_m(int mx, const QMat& W, const float* x, float* y, cudaStream_t s, int num_sms) {
  switch (mx) {
    case 1: return launch_gemv<1, R, CPL>(W, x, y, s, num_sms);
    case 2: return launch_gemv<2, R, CPL>(W, x, y, s, num_sms);
    case 3: return launch_gemv<3, R, CPL>(W, x, y, s, num_sms);
    default: return launch_gemv<4, R, CPL>(W, x, y, s, num_sms);
  }
}

template <int NT>
static int launch_gemv_mma(int mx, const QMat& W, const float* x, float* y, cudaStream_t s, int num_sms) {
  const size_t smem = (size_t)digit_image_bytes(mx, W.K);
  if (smem > 200 * 1024) return -1;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(k_gemv_mma<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return -1;
  const int ntiles = (W.N + 15) / 16;
  // few tiles: split K over the warps of one CTA per tile, so that about 16 warps per SM are
  // streaming (up to 16 warps per tile, at least one K block each); with two n-tiles (3-4
  // vectors) only while the tiles fit one wave, past that the grid-stride form measured faster
  int kw = 1;
  if (NT == 1 || ntiles <= num_sms)
    while (kw < 16 && 2 * kw <= W.K / 128 && ntiles * kw * 2 <= num_sms * 16) kw *= 2;
  if (kw > 1) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k_gemv_mma_sk<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return -1;
    // programmatic launch lets the next GEMV's CTAs start as these retire (~0.4 us per launch
    // at most shapes); with one vector at K = 8192 the early dependents measured slower
    if (NT == 1 && W.K >= 8192) k_gemv_mma_sk<NT><<<ntiles, 32 * kw, smem, s>>>(x, mx, W, y);
    else launch_pdl(k_gemv_mma_sk<NT>, dim3(ntiles), dim3(32 * kw), smem, s, x, mx, W, y);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
  }
  const int grid = std::min<int>((ntiles + 7) / 8, num_sms * 4);
  launch_pdl(k_gemv_mma<NT>, dim3(grid), dim3(256), smem, s, x, mx, W, y);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Kernel selection for the isolated GEMV: LLAMA_B128_GEMV=simt forces the CUDA-core kernel,
// otherwise the integer tensor-core kernel is used (N >= 16).
static bool gemv_use_mma(int N) {
  static int forced = -1;
  if (forced < 0) {
    const char* v = getenv("LLAMA_B128_GEMV");
    forced = (v && std::strcmp(v, "simt") == 0) ? 0 : 1;
  }
  return forced == 1 && N >= 16;
}

LE_API int llama_b128_gemv(const uint8_t* nibbles, const uint16_t* step_bf16, const uint16_t* min_bf16, int N, int K,
                           const float* x, int M, float* y, void* stream) {
  if (!nibbles || !step_bf16 || !min_bf16 || !x || !y) return -1;
  if (N < 1 || K < 128 || K % 128 != 0 || M < 1 || M > 8) return -1;
  // 16-byte vector loads of the nibble rows and of x
  if ((reinterpret_cast<uintptr_t>(nibbles) | reinterpret_cast<uintptr_t>(x)) & 15u) return -1;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  QMat W{nibbles, step_bf16, min_bf16, N, K};
  for (int m0 = 0; m0 < M; m0 += 4) {
    const int mx = std::min(4, M - m0);
    const float* xm = x + (size_t)m0 * K;
    float* ym = y + (size_t)m0 * N;
    int rc;
    if (gemv_use_mma(N)) {
      rc = mx <= 2 ? launch_gemv_mma<1>(mx, W, xm, ym, s, sms) : launch_gemv_mma<2>(mx, W, xm, ym, s, sms);
    } else if (N % 2 == 0) {
      rc = K >= 8192 ? launch_gemv_m<2, 8>(mx, W, xm, ym, s, sms) : launch_gemv_m<2, 2>(mx, W, xm, ym, s, sms);
    } else {
      rc = K >= 8192 ? launch_gemv_m<1, 8>(mx, W, xm, ym, s, sms) : launch_gemv_m<1, 2>(mx, W, xm, ym, s, sms);
    }
    if (rc != 0) return -1;
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------
// Isolated tensor-core GEMM (the batched path's kernel on a caller's matrix): builds the weight
// records and the activation image in temporary device buffers, runs k_tc_gemm, waits for it and
// frees the buffers.  For tests and measurements, not for a serving loop.
// ---------------------------------------------------------------------------------------------
LE_API int llama_b128_gemm(const uint8_t* nibbles, const uint16_t* step_bf16, const uint16_t* min_bf16, int N, int K,
                           const float* x, int M, float* y, void* stream) {
  using namespace le::tc;
  if (!nibbles || !step_bf16 || !min_bf16 || !x || !y) return -1;
  if (N < 1 || K < 2048 || K % 2048 != 0 || K > 8192 || M < 1 || M > 4096) return -1;
  if ((reinterpret_cast<uintptr_t>(nibbles) | reinterpret_cast<uintptr_t>(x)) & 15u) return -1;
  int dev = 0, sms = 148;
  cudaDeviceProp prop{};
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return -1;
  if (prop.major != 10) return -1;
  sms = prop.multiProcessorCount;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int kb = K / 128, tiles = (N + kM - 1) / kM, tok_tiles = (M + kTok - 1) / kTok;
  uint8_t *recs = nullptr, *img = nullptr;
  uint32_t* err = nullptr;
  int rc = -1;
  const size_t rec_bytes = (size_t)tiles * kb * tc::kRecBytes, img_bytes = (size_t)tok_tiles * kb * kImgBytes;
  if (cudaMalloc(&recs, rec_bytes) == cudaSuccess && cudaMalloc(&img, img_bytes) == cudaSuccess &&
      cudaMalloc(&err, 16) == cudaSuccess) {
    static bool attr = false;
    if (!attr)
      attr = cudaFuncSetAttribute(k_tc_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<1>::kSmemBytes) ==
                 cudaSuccess &&
             cudaFuncSetAttribute(k_tc_gemm<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<2>::kSmemBytes) ==
                 cudaSuccess;
    // the unit form the engine's steps would take for this shape (no K splits here)
    const TcPlan pl = tc_plan(sms, tiles, kb, tok_tiles, 1);
    const int P = pl.P;
    cudaMemsetAsync(recs, 0, rec_bytes, s);
    cudaMemsetAsync(img, 0, img_bytes, s);
    cudaMemsetAsync(err, 0, 16, s);
    QMat W{nibbles, step_bf16, min_bf16, N, K};
    k_tc_repack<<<sms * 8, 256, 0, s>>>(W, recs, 0, kM, 0, 1);
    k_tc_stage<false><<<dim3(M, K / 2048), 256, 0, s>>>(const_cast<float*>(x), K, nullptr, 0, 0, nullptr, K, img);
    Args A{};
    A.recs = recs;
    A.img = img;
    A.tiles = tiles;
    A.kb_total = kb;
    A.img_tiles = tok_tiles;
    A.tok_tiles = pl.groups;
    A.splits = 1;
    A.kb_split = kb;
    A.T = M;
    A.N = N;
    A.out = y;
    A.ldo = N;
    A.error = err;
    A.wait_ns = kWaitNs;
    // diagnostics: $LLAMA_B128_GEMM_TRACE names a file that receives CTA 0's pipeline events
    const char* trace_path = getenv("LLAMA_B128_GEMM_TRACE");
    unsigned long long* trace = nullptr;
    const size_t trace_bytes = (size_t)kTraceEvents * kTraceBlocks * 8;
    if (trace_path && cudaMalloc(&trace, trace_bytes) == cudaSuccess) {
      cudaMemsetAsync(trace, 0, trace_bytes, s);
      A.trace = trace;
    }
    const int grid = std::min(tiles * A.tok_tiles, sms);
    if (P == 2)
      k_tc_gemm<2><<<grid, Geo<2>::kThreads, Geo<2>::kSmemBytes, s>>>(A);
    else
      k_tc_gemm<1><<<grid, Geo<1>::kThreads, Geo<1>::kSmemBytes, s>>>(A);
    if (trace) {
      std::vector<unsigned long long> h(trace_bytes / 8);
      if (cudaMemcpyAsync(h.data(), trace, trace_bytes, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
          cudaStreamSynchronize(s) == cudaSuccess) {
        if (FILE* f = fopen(trace_path, "wb")) {
          fwrite(h.data(), 8, h.size(), f);
          fclose(f);
        }
      }
      cudaFree(trace);
    }
    uint32_t herr = 1;
    if (attr && cudaGetLastError() == cudaSuccess &&
        cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
        cudaStreamSynchronize(s) == cudaSuccess && herr == 0)
      rc = 0;
  }
  cudaStreamSynchronize(s);
  if (recs) cudaFree(recs);
  if (img) cudaFree(img);
  if (err) cudaFree(err);
  return rc;
}

// ---------------------------------------------------------------------------------------------
// Greedy argmax that allocates nothing
//
// For callers that must not allocate device memory once they are running: serving processes
// that reserve their whole memory budget at start-up, and latency-critical decode loops, where a
// cudaMalloc can synchronise the device and stall every stream.  The per-CTA candidates live in
// a fixed file-scope device array instead of caller- or engine-allocated scratch.  Every GPU
// that loads this library holds the array (8 KB) until the process exits.
// ---------------------------------------------------------------------------------------------
namespace {
constexpr int kNoAllocParts = 1024;               // candidate slots in the static scratch array
constexpr int kNoAllocPerThread = 64;             // at most this many logits per thread
constexpr long long kNoAllocMaxN = (long long)kNoAllocParts * le::kThreads * kNoAllocPerThread;  // 16,777,216

static __device__ __align__(256) le::ArgmaxPart g_argmax_scratch[kNoAllocParts];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_argmax_scratch, per device ordinal
}  // namespace

LE_API int llama_b128_argmax_noalloc(const float* logits, int n, int32_t* out_index, void* stream) {
  if (!logits || !out_index || n < 1) return -1;
  if ((long long)n > kNoAllocMaxN) return -2;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  void* scratch = nullptr;
  {
    // once per device, with that device current: the host-side symbol is only a stand-in, the
    // kernels need the device address
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p) return -1;
      g_noalloc_addr[dev] = p;
    }
    scratch = g_noalloc_addr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  le::ArgmaxPart* part = static_cast<le::ArgmaxPart*>(scratch);
  // every candidate slot the finish kernel reads is written by this call: nothing to clear
  const long long per_part = (long long)le::kThreads * 4;
  const int parts = (int)std::min<long long>(kNoAllocParts, ((long long)n + per_part - 1) / per_part);
  le::k_argmax_rows<<<parts, le::kThreads, 0, s>>>(logits, n, part);
  le::k_argmax_finish<<<1, 1024, 0, s>>>(part, parts, out_index, nullptr, nullptr, 0);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
