// Module preamble of the LTC layer, fused: LayerNorm over D followed by the
// input affine map (reference ltc.py:259 and ltc.py:266):
//   xhat = (x - mean) * rstd,  rstd = 1/sqrt(var + eps)     (biased variance)
//   y    = (xhat * ln_w + ln_b) * in_w + in_b
// Forward: one warp per row (b,t), the row held in registers (D <= 32*VPL),
// two-pass mean/variance; writes y and (mean, rstd) per row.
// Backward: one warp per row recomputes xhat and produces dx; the four column
// gradients (in_w, in_b, ln_w, ln_b) are accumulated per warp in registers,
// reduced across the CTA's warps in a fixed order into one partial slab per
// CTA, and summed over CTAs in a fixed order by a second kernel.
#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace ltc {

namespace {

constexpr int kWarps = 8;  // rows per CTA pass

template <int VPL>
__global__ void __launch_bounds__(kWarps * 32) preamble_fwd_kernel(PreambleArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = a.D;
  float w[VPL], b[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int d = lane + 32 * k;
    const bool ok = d < D;
    const float lw = ok ? a.ln_w[d] : 0.f, lb = ok ? a.ln_b[d] : 0.f;
    const float iw = ok ? a.in_w[d] : 0.f, ib = ok ? a.in_b[d] : 0.f;
    w[k] = lw * iw;       // y = xhat * (lw*iw) + (lb*iw + ib)
    b[k] = fmaf(lb, iw, ib);
  }
  const float invD = 1.0f / (float)D;
  for (long long row = (long long)blockIdx.x * kWarps + warp; row < a.rows; row += (long long)gridDim.x * kWarps) {
    const float* xr = a.x + row * D;
    float v[VPL];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int d = lane + 32 * k;
      v[k] = d < D ? xr[d] : 0.f;
      s += v[k];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * invD;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int d = lane + 32 * k;
      const float c = d < D ? v[k] - mean : 0.f;
      q = fmaf(c, c, q);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = rsqrtf(q * invD + a.eps);
    float* yr = a.y + row * D;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) yr[d] = fmaf((v[k] - mean) * rstd, w[k], b[k]);
    }
    if (lane == 0) {
      a.stats[2 * row] = mean;
      a.stats[2 * row + 1] = rstd;
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(kWarps * 32) preamble_bwd_kernel(PreambleArgs a) {
  __shared__ float red[kWarps][32 * VPL];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = a.D;
  float lw[VPL], lb[VPL], iw[VPL];
  float g_iw[VPL], g_ib[VPL], g_lw[VPL], g_lb[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int d = lane + 32 * k;
    const bool ok = d < D;
    lw[k] = ok ? a.ln_w[d] : 0.f;
    lb[k] = ok ? a.ln_b[d] : 0.f;
    iw[k] = ok ? a.in_w[d] : 0.f;
    g_iw[k] = g_ib[k] = g_lw[k] = g_lb[k] = 0.f;
  }
  const float invD = 1.0f / (float)D;
  for (long long row = (long long)blockIdx.x * kWarps + warp; row < a.rows; row += (long long)gridDim.x * kWarps) {
    const float* xr = a.x + row * D;
    const float* gr = a.dy + row * D;
    const float mean = a.stats[2 * row], rstd = a.stats[2 * row + 1];
    float xh[VPL], u[VPL];
    float su = 0.f, sux = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int d = lane + 32 * k;
      const bool ok = d < D;
      const float dy = ok ? gr[d] : 0.f;
      xh[k] = ok ? (xr[d] - mean) * rstd : 0.f;
      const float xn = fmaf(xh[k], lw[k], lb[k]);  // LayerNorm output
      g_iw[k] = fmaf(dy, xn, g_iw[k]);
      g_ib[k] += dy;
      const float dxn = dy * iw[k];
      g_lw[k] = fmaf(dxn, xh[k], g_lw[k]);
      g_lb[k] += dxn;
      u[k] = dxn * lw[k];  // dL/dxhat
      su += u[k];
      sux = fmaf(u[k], xh[k], sux);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      su += __shfl_xor_sync(0xffffffffu, su, o);
      sux += __shfl_xor_sync(0xffffffffu, sux, o);
    }
    const float mu_u = su * invD, mu_ux = sux * invD;
    float* dxr = a.dx + row * D;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) dxr[d] = rstd * (u[k] - mu_u - xh[k] * mu_ux);
    }
  }
  // fixed-order reduction of the column gradients over the CTA's warps, one
  // gradient vector at a time (shared memory holds kWarps rows of 32*VPL)
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const float gv = j == 0 ? g_iw[k] : j == 1 ? g_ib[k] : j == 2 ? g_lw[k] : g_lb[k];
      red[warp][lane + 32 * k] = gv;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += kWarps * 32) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += red[w][c];
      a.part[((long long)blockIdx.x * 4 + j) * D + c] = s;
    }
    __syncthreads();
  }
}

__global__ void preamble_finish_kernel(PreambleArgs a, int nblocks) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 4 * a.D; i += gridDim.x * blockDim.x) {
    const int j = i / a.D, c = i % a.D;
    float s = 0.f;
    for (int bI = 0; bI < nblocks; ++bI) s += a.part[((long long)bI * 4 + j) * a.D + c];
    float* out = j == 0 ? a.g_in_w : j == 1 ? a.g_in_b : j == 2 ? a.g_ln_w : a.g_ln_b;
    out[c] = s;
  }
}

int vpl_of(int D) {
  const int v = (D + 31) / 32;
  return v <= 4 ? 4 : v <= 8 ? 8 : v <= 16 ? 16 : 32;
}

}  // namespace

int preamble_blocks(long long rows, int num_sms) {
  const long long need = (rows + kWarps - 1) / kWarps;
  const long long cap = 4LL * num_sms;
  return (int)(need < cap ? (need > 0 ? need : 1) : cap);
}

cudaError_t launch_preamble_fwd(const PreambleArgs& a, int num_sms, cudaStream_t st) {
  const int blocks = preamble_blocks(a.rows, num_sms);
  switch (vpl_of(a.D)) {
    case 4: preamble_fwd_kernel<4><<<blocks, kWarps * 32, 0, st>>>(a); break;
    case 8: preamble_fwd_kernel<8><<<blocks, kWarps * 32, 0, st>>>(a); break;
    case 16: preamble_fwd_kernel<16><<<blocks, kWarps * 32, 0, st>>>(a); break;
    default: preamble_fwd_kernel<32><<<blocks, kWarps * 32, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_preamble_bwd(const PreambleArgs& a, int num_sms, cudaStream_t st) {
  const int blocks = preamble_blocks(a.rows, num_sms);
  switch (vpl_of(a.D)) {
    case 4: preamble_bwd_kernel<4><<<blocks, kWarps * 32, 0, st>>>(a); break;
    case 8: preamble_bwd_kernel<8><<<blocks, kWarps * 32, 0, st>>>(a); break;
    case 16: preamble_bwd_kernel<16><<<blocks, kWarps * 32, 0, st>>>(a); break;
    default: preamble_bwd_kernel<32><<<blocks, kWarps * 32, 0, st>>>(a); break;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  preamble_finish_kernel<<<(4 * a.D + 255) / 256, 256, 0, st>>>(a, blocks);
  return cudaGetLastError();
}

}  // namespace ltc
