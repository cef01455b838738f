// Shared device helpers for the sm_100a kernels of the block-128 4-bit engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define LE_MAX_SEQ_LEN 8192  // MAX_SEQ_LEN, src/llama_engine.cpp:26
#define LE_HEAD_DIM 64       // head_dim fixed by the reference's attention loops (:978, :1010, :1017)

// One quantised matrix on the device, in the LLM4S128 layout: row n owns K/128 consecutive
// blocks; a block is 64 bytes of nibbles (low nibble = even element) and one bf16 step and
// one bf16 min (src/llama_engine.cpp:156-180).
struct QMat {
  const uint8_t* nib;    // [N][K/2]
  const uint16_t* step;  // [N][K/128] bf16 bits
  const uint16_t* mn;    // [N][K/128] bf16 bits
  int N, K;
};

// bf16 -> fp32 is a 16-bit shift (src/llama_engine.cpp:28-33).
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// Balanced base-256 digits of a fixed-point integer |X| < 2^29: the bytes of the result, read as
// s8, are d0..d3 with X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3 and every d in [-128, 127].  (Adding 128
// to every byte position and then flipping each byte's top bit is the same as taking the digit
// d = ((X + 128) & 255) - 128 and carrying (X - d) >> 8 to the next position.)
__device__ __forceinline__ uint32_t balanced_digits(int X) {
  return ((uint32_t)X + 0x80808080u) ^ 0x80808080u;
}
// Byte transpose of four digit words: plane p of the result holds byte p of d0, d1, d2, d3 (in
// that byte order).
__device__ __forceinline__ void digit_planes(uint32_t d0, uint32_t d1, uint32_t d2, uint32_t d3, uint32_t (&pl)[4]) {
  const uint32_t t0 = __byte_perm(d0, d1, 0x5140), t1 = __byte_perm(d0, d1, 0x7362);
  const uint32_t t2 = __byte_perm(d2, d3, 0x5140), t3 = __byte_perm(d2, d3, 0x7362);
  pl[0] = __byte_perm(t0, t2, 0x5410);
  pl[1] = __byte_perm(t0, t2, 0x7632);
  pl[2] = __byte_perm(t1, t3, 0x5410);
  pl[3] = __byte_perm(t1, t3, 0x7632);
}

// Programmatic dependent launch (kernels of one batched step, launched with the programmatic
// stream-serialisation attribute): the kernel lets the next one in the stream be scheduled as
// soon as all of its CTAs are running, then waits until the previous kernel has completed and
// its memory is visible.  Without the attribute both instructions are no-ops.  A kernel must
// not touch memory that an earlier kernel of the stream writes or reads before the wait.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_begin() {
  grid_dep_launch();
  grid_dep_wait();
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 16-byte load of weights: read once per token, so keep them out of L1.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Exact float value of a 4-bit code held in the low bits of `q` (q < 16): the bit pattern
// 0x4B000000 | q is 2^23 + q, and subtracting 2^23 is exact.
__device__ __forceinline__ float nib_to_f32(uint32_t q) {
  return __uint_as_float(0x4B000000u | q) - 8388608.0f;
}

// Block-wide sum for blockDim.x threads (a multiple of 32, at most 1024).  `red` must hold 32
// floats of shared memory.  Every thread receives the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}
