// Block-128 4-bit GEMV on the integer tensor-core path (mma.sync m16n8k32, u8 x s8 -> s32).
//
// The factored form of the reference GEMV (src/llama_engine.cpp:231-232, 315-319),
//     y_n = sum_b ( min_nb * xs_b + step_nb * sum_{k in b} q_nk * x_k ),
// needs the exact 4-bit codes q (0..15) times the activations.  Here the codes go into the
// tensor core unchanged as u8, and each 128-block of the fp32 activation vector is written as a
// 30-bit fixed-point integer split into four balanced base-256 digits:
//     x_k ~= 2^-e_b * X_k,   X_k = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3,   d_i in [-128, 127],
// with e_b chosen so that max_k |x_k| * 2^e_b < 2^29.  The four digit planes are four columns
// of the MMA's B operand (N = 8 holds two activation vectors), so one MMA returns the exact
// integer sums  C_i = sum_k q_k d_ik  for a 16-row tile.  Per block the tile's rows then add
//     step * 2^-e_b * (((C3 * 256 + C2) * 256 + C1) * 256 + C0)  +  min * xs_b
// in fp32.  The only rounding inside a block is the 2^-30-relative fixed-point step of x and
// the final fp32 combination, so the result matches an fp32 loop to ~1e-7 relative.
//
// Operand layout.  A warp owns a tile of 16 rows.  For block b, lane (g, t) (g = lane/4,
// t = lane%4) loads bytes [16t, 16t+16) of rows g and g+8 of the block (two coalesced 512-byte
// warp loads).  Its u32 word i (i = 0..3) holds codes 32t+8i .. 32t+8i+7 of the block:
//   a0 = word & 0x0F0F0F0F (row g, codes 32t+8i+{0,2,4,6}), a2 = (word >> 4) & 0x0F0F0F0F
//   (codes +{1,3,5,7}); a1 / a3 likewise from row g+8.  MMA i of the block covers the 32 codes
// {32t+8i+m}; the B fragments are written in the same permuted K order by stage_digits().
#pragma once

#include "common.cuh"

namespace le {

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory image of MX activation vectors for the MMA path.
//   bfrag : [nb][4 (MMA i)][NT (n-tile)][32 lanes] uint2, NT = (MX+1)/2
//   bsum  : [MX][nb]  fp32 block sums (compute_x_block_sums, src/llama_engine.cpp:496-521)
//   escl  : [MX][nb]  2^-e_b
struct DigitImage {
  uint2* bfrag;
  float* bsum;
  float* escl;
};

__host__ __device__ constexpr int digit_image_bytes(int MX, int K) {
  return (K / 128) * 4 * ((MX + 1) / 2) * 32 * 8 + 2 * MX * (K / 128) * 4;
}

// Builds the digit image from MX fp32 vectors xs[m*K + k] already in shared memory.
// Must be called by the whole CTA; ends with __syncthreads().
__device__ __forceinline__ void stage_digits(const float* xs, int MX, int K, DigitImage img) {
  const int nb = K / 128, NT = (MX + 1) / 2;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  // 1) per-block sum and exponent: one warp per (m, b)
  for (int mb = wid; mb < MX * nb; mb += nw) {
    const float4 v = *reinterpret_cast<const float4*>(xs + (size_t)mb * 128 + lane * 4);
    float s = (v.x + v.y) + (v.z + v.w);
    float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    s = warp_sum(s);
    a = warp_max(a);
    if (lane == 0) {
      // a < 2^ex with ex from the exponent field (denormals bounded by 2^-126)
      const int ex = max((int)((__float_as_uint(a) >> 23) & 0xFFu), 1) - 126;
      const int e = min(29 - ex, 126);
      img.bsum[mb] = s;
      img.escl[mb] = (a > 0.0f) ? __uint_as_float((uint32_t)(127 - e) << 23) : 0.0f;
    }
  }
  // Zero the unused half of the last n-tile when MX is odd (lanes 16..31 of n-tile NT-1).
  if (MX & 1) {
    for (int u = threadIdx.x; u < nb * 4 * 16; u += blockDim.x) {
      const int bi = u >> 4, l = 16 + (u & 15);
      img.bfrag[((size_t)bi * NT + (NT - 1)) * 32 + l] = make_uint2(0u, 0u);
    }
  }
  __syncthreads();
  // 2) digits: one unit = (m, b, i, t, h) covering codes n = 32t + 8i + 2j + h, j = 0..3
  const int units = MX * nb * 32;
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int h = u & 1, t = (u >> 1) & 3, i = (u >> 3) & 3, b = (u >> 5) % nb, m = (u >> 5) / nb;
    const float es = img.escl[m * nb + b];
    const int e = es > 0.0f ? 127 - (int)(__float_as_uint(es) >> 23) : 0;
    const float up = __uint_as_float((uint32_t)(e + 127) << 23);  // 2^e
    uint32_t dg[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float xv = xs[(size_t)m * K + b * 128 + 32 * t + 8 * i + 2 * j + h];
      dg[j] = balanced_digits(es > 0.0f ? __float2int_rn(xv * up) : 0);
    }
    uint32_t plane[4];
    digit_planes(dg[0], dg[1], dg[2], dg[3], plane);
    const int jt = m >> 1;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int L = ((m & 1) * 4 + p) * 4 + t;
      uint32_t* dst = reinterpret_cast<uint32_t*>(&img.bfrag[(((size_t)b * 4 + i) * NT + jt) * 32 + L]);
      dst[h] = plane[p];
    }
  }
  __syncthreads();
}

// One output row-pair result per thread: lanes with t in {0, 2} own (rows g, g+8) of sequence
// 2*j + t/2 for each n-tile j.
template <int NT>
struct TileAcc {
  float y[NT][2];
};

// Accumulates the tile (16 rows starting at row0 of W) over K blocks [b0, b1).  Block b+1's
// nibbles are requested before block b is computed; with kScalesAhead its scales too (pays when
// few warps share an SM, as in the split-K form, and costs when many do).
template <int NT, bool kScalesAhead>
__device__ __forceinline__ void mma_tile(const QMat& W, int row0, const DigitImage& img, int MX, TileAcc<NT>& acc,
                                         int b0 = 0, int b1 = -1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nb = W.K >> 7;
  const uint8_t* ra = W.nib + (size_t)(row0 + g) * (W.K >> 1) + 16 * t;
  const uint8_t* rb = ra + (size_t)8 * (W.K >> 1);
  const uint16_t* sa = W.step + (size_t)(row0 + g) * nb;
  const uint16_t* ma = W.mn + (size_t)(row0 + g) * nb;
  const uint16_t* sb = sa + (size_t)8 * nb;
  const uint16_t* mb = ma + (size_t)8 * nb;
  const bool owner = (t & 1) == 0;
  const int seq_off = t >> 1;
#pragma unroll
  for (int j = 0; j < NT; ++j) acc.y[j][0] = acc.y[j][1] = 0.0f;

  if (b1 < 0) b1 = nb;
  if (b0 >= b1) return;
  auto scales = [&](int b, float (&sc)[4]) {
    sc[0] = sc[1] = sc[2] = sc[3] = 0.f;
    if (owner) {
      sc[0] = bf16_bits_to_f32(__ldg(sa + b));
      sc[1] = bf16_bits_to_f32(__ldg(ma + b));
      sc[2] = bf16_bits_to_f32(__ldg(sb + b));
      sc[3] = bf16_bits_to_f32(__ldg(mb + b));
    }
  };
  uint4 wa = ld_stream_u4(ra + (size_t)b0 * 64), wb = ld_stream_u4(rb + (size_t)b0 * 64);
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
  if (kScalesAhead) scales(b0, sc);
  for (int b = b0; b < b1; ++b) {
    uint4 na = wa, nbw = wb;
    float nsc[4] = {sc[0], sc[1], sc[2], sc[3]};
    if (b + 1 < b1) {
      na = ld_stream_u4(ra + (size_t)(b + 1) * 64);
      nbw = ld_stream_u4(rb + (size_t)(b + 1) * 64);
      if (kScalesAhead) scales(b + 1, nsc);
    }
    int c[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0;
    const uint2* bf = img.bfrag + (size_t)b * 4 * NT * 32 + lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t xa = i == 0 ? wa.x : i == 1 ? wa.y : i == 2 ? wa.z : wa.w;
      const uint32_t xb = i == 0 ? wb.x : i == 1 ? wb.y : i == 2 ? wb.z : wb.w;
      const uint32_t a0 = xa & 0x0F0F0F0Fu, a2 = (xa >> 4) & 0x0F0F0F0Fu;
      const uint32_t a1 = xb & 0x0F0F0F0Fu, a3 = (xb >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint2 bq = bf[(i * NT + j) * 32];
        mma_u8s8(c[j], a0, a1, a2, a3, bq.x, bq.y);
      }
    }
    if (!kScalesAhead) scales(b, sc);
    // epilogue of block b: lanes t and t^1 hold digit planes {0,1} and {2,3}; each lane folds its
    // pair in int32 (|C| <= 128 * 15 * 128 < 2^18, so |C_even + 256 C_odd| < 2^27 is exact) and
    // one shuffle per row brings the high pair to the owner lane
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int x0 = c[j][0] + 256 * c[j][1], x1 = c[j][2] + 256 * c[j][3];
      const int h0 = __shfl_xor_sync(0xffffffffu, x0, 1);
      const int h1 = __shfl_xor_sync(0xffffffffu, x1, 1);
      const int m = 2 * j + seq_off;
      if (owner && m < MX) {
        const float es = img.escl[m * nb + b], xsb = img.bsum[m * nb + b];
        const float v0 = fmaf((float)h0, 65536.0f, (float)x0);
        const float v1 = fmaf((float)h1, 65536.0f, (float)x1);
        acc.y[j][0] += fmaf(sc[0] * es, v0, sc[1] * xsb);
        acc.y[j][1] += fmaf(sc[2] * es, v1, sc[3] * xsb);
      }
    }
    wa = na;
    wb = nbw;
#pragma unroll
    for (int q = 0; q < 4; ++q) sc[q] = nsc[q];
  }
}

}  // namespace le

namespace le {

// Isolated GEMV on the MMA path: y[m][n] = W[n,:] . x[m,:] for MX = 1..4 vectors.  Each warp
// processes 16-row tiles (grid-stride); rows past N are clamped on load and never stored.
template <int NT>
__global__ void __launch_bounds__(256) k_gemv_mma(const float* __restrict__ x, int MX, QMat W, float* __restrict__ y) {
  extern __shared__ float4 smem4[];
  const int nb = W.K / 128;
  DigitImage img;
  img.bfrag = reinterpret_cast<uint2*>(smem4);
  img.bsum = reinterpret_cast<float*>(img.bfrag + (size_t)nb * 4 * NT * 32);
  img.escl = img.bsum + MX * nb;
  grid_dep_wait();  // x (and y) may belong to the previous kernel of the stream
  stage_digits(x, MX, W.K, img);
  grid_dep_launch();  // the next kernel's CTAs may take SM room as this grid's CTAs retire
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ntiles = (W.N + 15) / 16;
  const int warps = blockDim.x >> 5;
  for (int tile = blockIdx.x * warps + (threadIdx.x >> 5); tile < ntiles; tile += gridDim.x * warps) {
    int row0 = tile * 16;
    QMat Wt = W;
    if (row0 + 16 > W.N) row0 = W.N - 16;  // N >= 16 is required by the launcher
    TileAcc<NT> acc;
    mma_tile<NT, false>(Wt, row0, img, MX, acc);
    if ((t & 1) == 0) {
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int m = 2 * j + (t >> 1);
        if (m < MX) {
          const int r0 = row0 + g, r1 = row0 + g + 8;
          if (r0 >= tile * 16) y[(size_t)m * W.N + r0] = acc.y[j][0];
          if (r1 >= tile * 16) y[(size_t)m * W.N + r1] = acc.y[j][1];
        }
      }
    }
  }
}


// Split-K form for matrices with few 16-row tiles (N up to a few thousand rows), where one warp
// per tile would leave most SMs idle and walk every K block in series: one CTA per tile, its KW
// warps take consecutive block ranges, and the CTA adds the KW partial rows in shared memory in
// warp order.  The digit image is staged by every CTA, as in k_gemv_mma.
template <int NT>
__global__ void __launch_bounds__(512) k_gemv_mma_sk(const float* __restrict__ x, int MX, QMat W,
                                                      float* __restrict__ y) {
  extern __shared__ float4 smem4[];
  __shared__ float red[16][4][16];  // [warp][sequence][row]
  const int nb = W.K / 128;
  DigitImage img;
  img.bfrag = reinterpret_cast<uint2*>(smem4);
  img.bsum = reinterpret_cast<float*>(img.bfrag + (size_t)nb * 4 * NT * 32);
  img.escl = img.bsum + MX * nb;
  grid_dep_wait();  // x (and y) may belong to the previous kernel of the stream
  stage_digits(x, MX, W.K, img);
  const int KW = blockDim.x >> 5, w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x;
  int row0 = tile * 16;
  if (row0 + 16 > W.N) row0 = W.N - 16;  // N >= 16 is required by the launcher
  const int per = (nb + KW - 1) / KW;
  const int b0 = min(nb, w * per), b1 = min(nb, b0 + per);
  TileAcc<NT> acc;
#pragma unroll
  for (int j = 0; j < NT; ++j) acc.y[j][0] = acc.y[j][1] = 0.0f;
  mma_tile<NT, NT == 1>(W, row0, img, MX, acc, b0, b1);
  grid_dep_launch();  // only the reduction and the store remain
  if ((t & 1) == 0) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int m = 2 * j + (t >> 1);
      if (m < MX) {
        red[w][m][g] = acc.y[j][0];
        red[w][m][g + 8] = acc.y[j][1];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < 16 * MX) {
    const int m = threadIdx.x >> 4, r = threadIdx.x & 15;
    float v = 0.0f;
    for (int k = 0; k < KW; ++k) v += red[k][m][r];
    if (row0 + r >= tile * 16) y[(size_t)m * W.N + row0 + r] = v;
  }
}

}  // namespace le
