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
