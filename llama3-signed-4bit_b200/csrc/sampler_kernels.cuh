// Temperature sampling support (sample_top_p, src/llama_engine.cpp:794-806): the logits are
// scaled by 1/temperature, exponentiated against their maximum and normalised, in place, so that
// llama_engine_get_logits() afterwards returns probabilities exactly as in the reference.
#pragma once

namespace le {

__global__ void k_scale_max(float* __restrict__ l, int n, float inv_t, float* __restrict__ part) {
  __shared__ float red[32];
  float m = -1e30f;  // the reference's running maximum starts at -1e30 (:797)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = l[i] * inv_t;
    l[i] = v;
    if (v > m) m = v;
  }
  m = block_max(m, red);
  if (threadIdx.x == 0) part[blockIdx.x] = m;
}

__global__ void k_exp_sum(float* __restrict__ l, int n, const float* __restrict__ part_max, int nparts,
                          float* __restrict__ part_sum) {
  __shared__ float red[32];
  __shared__ float s_max;
  if (threadIdx.x < 32) {
    float m = -1e30f;
    for (int i = threadIdx.x; i < nparts; i += 32) m = fmaxf(m, part_max[i]);
    m = warp_max(m);
    if (threadIdx.x == 0) s_max = m;
  }
  __syncthreads();
  const float mx = s_max;
  float s = 0.0f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float e = expf(l[i] - mx);
    l[i] = e;
    s += e;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) part_sum[blockIdx.x] = s;
}

__global__ void k_normalize(float* __restrict__ l, int n, const float* __restrict__ part_sum, int nparts) {
  __shared__ float s_inv;
  if (threadIdx.x < 32) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < nparts; i += 32) s += part_sum[i];
    s = warp_sum(s);
    if (threadIdx.x == 0) s_inv = 1.0f / s;
  }
  __syncthreads();
  const float inv = s_inv;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) l[i] *= inv;
}

// The 64 candidates of sample_top_p (src/llama_engine.cpp:808-822), exactly as the reference's
// walk builds them: the list starts as ids 0..63 in index order, then every later id whose
// probability exceeds the list's last entry is inserted after the last entry that is >= it
// (shifting the rest down and dropping the last).  The walk is sequential by nature; warp 0
// replays it from shared memory, one 32-id chunk at a time (a ballot finds the ids that beat the
// current last entry; each insertion is a warp-wide ballot and shift, list entry j held by lane
// j / 2), while warps 1..7 stage the next 4096 probabilities.  n >= 64.  Writes ids then values.
constexpr int kTopkTile = 4096;
__global__ void __launch_bounds__(256) k_topk64_walk(const float* __restrict__ p, int n, int32_t* __restrict__ out_ids,
                                                     float* __restrict__ out_vals) {
  __shared__ float tile[2][kTopkTile];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (n - 64 + kTopkTile - 1) / kTopkTile;  // ids 64 .. n-1
  auto load = [&](int t, int b) {  // warps 1..7
    const int base = 64 + t * kTopkTile;
    for (int i = threadIdx.x - 32; i < kTopkTile; i += blockDim.x - 32)
      tile[b][i] = base + i < n ? p[base + i] : 0.0f;
  };
  float v0 = 0.0f, v1 = 0.0f;
  int i0 = 0, i1 = 0;
  if (warp == 0) {
    i0 = 2 * lane;
    i1 = 2 * lane + 1;
    v0 = p[i0];
    v1 = p[i1];
  } else if (ntiles > 0) {
    load(0, 0);
  }
  __syncthreads();
  for (int t = 0; t < ntiles; ++t) {
    const int b = t & 1;
    if (warp != 0) {
      if (t + 1 < ntiles) load(t + 1, b ^ 1);
    } else {
      const int base = 64 + t * kTopkTile;
      const int cnt = min(kTopkTile, n - base);
      for (int c0 = 0; c0 < cnt; c0 += 32) {
        const float v = c0 + lane < cnt ? tile[b][c0 + lane] : 0.0f;
        const bool valid = c0 + lane < cnt;
        unsigned done = 0u;  // lanes (ids) of this chunk already walked past
        while (true) {
          const float last = __shfl_sync(0xffffffffu, v1, 31);
          const unsigned m = __ballot_sync(0xffffffffu, valid && v > last) & ~done;
          if (m == 0u) break;
          const int src = __ffs(m) - 1;  // the next id in index order that beats the last entry
          done |= (2u << src) - 1u;      // ids up to src are walked past
          const float w = __shfl_sync(0xffffffffu, v, src);
          const int wi = base + c0 + src;
          // q = 1 + the last list position holding a value >= w (0 if none)
          const int hp = v1 >= w ? 2 * lane + 1 : (v0 >= w ? 2 * lane : -1);
          const int q = __reduce_max_sync(0xffffffffu, hp) + 1;
          const float up1 = __shfl_up_sync(0xffffffffu, v1, 1);
          const int upi1 = __shfl_up_sync(0xffffffffu, i1, 1);
          const int p0 = 2 * lane, p1 = 2 * lane + 1;
          float n0 = v0, n1 = v1;
          int ni0 = i0, ni1 = i1;
          if (p1 > q) { n1 = v0; ni1 = i0; } else if (p1 == q) { n1 = w; ni1 = wi; }
          if (p0 > q) { n0 = up1; ni0 = upi1; } else if (p0 == q) { n0 = w; ni0 = wi; }
          v0 = n0; v1 = n1; i0 = ni0; i1 = ni1;
        }
      }
    }
    __syncthreads();
  }
  if (warp == 0) {
    out_ids[2 * lane] = i0;
    out_ids[2 * lane + 1] = i1;
    out_vals[2 * lane] = v0;
    out_vals[2 * lane + 1] = v1;
  }
}

static bool softmax_in_place(Engine* E, float temperature) {
  const int parts = std::min<int>(E->num_sms * 2, (E->vocab + kThreads - 1) / kThreads);
  const float inv_t = 1.0f / temperature;  // :794
  k_scale_max<<<parts, kThreads, 0, E->stream>>>(E->logits, E->vocab, inv_t, E->red);
  k_exp_sum<<<parts, kThreads, 0, E->stream>>>(E->logits, E->vocab, E->red, parts, E->red + 1024);
  k_normalize<<<parts, kThreads, 0, E->stream>>>(E->logits, E->vocab, E->red + 1024, parts);
  LE_CK(cudaGetLastError());
  E->argmax_valid = false;
  E->logits_on_host_fresh = false;
  return true;
}

}  // namespace le
