// Shared device helpers for the LTC solver kernels (sm_100a).
//
// Conventions used by every kernel in this library
// ------------------------------------------------
// * fp32 everywhere.  Recurrent matrices are (H, H) row-major indexed
//   [pre p, post q]; sensory matrices are (D, H) indexed [input d, post q].
// * A sigmoid gate  act = 1 / (1 + exp(-sigma * (v - mu)))  is evaluated from a
//   per-synapse "gate pack" holding the half-scale constants
//   (sh, nh) = (sigma/2, -sigma*mu/2), so that z/2 = sh*v + nh, as
//   act = 0.5 + 0.5 * tanh(z/2) with the hardware tanh.approx (one MUFU op).
//   The forward kernels fold the 0.5 terms into sums of the weights.
// * Saved forward state for the backward pass:
//     V[n][b][h], n = t*U + k, n in [0, T*U]: the input of unfold k at step t
//       (V[T*U] is the final state);
//     R[n][b][h], n in [0, T*U): 1 / (cm_t + gleak + den + eps) of that unfold.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>


namespace ltc {

// ---- checked build (-DLTC_CHECKED) ---------------------------------------------
// LTC_CHECK(cond, site) records an index that breaks its bound instead of trapping:
// the failing count and the first failing site go into a per-file device word pair,
// which the host gathers with ltc_check_errors() after a sync.  The caller of the
// check skips the access itself (LTC_CHECKED_SKIP).  In the normal build every check
// compiles to nothing.
#ifdef LTC_CHECKED
void register_check_reader(int (*reader)(int* count, int* site));
static __device__ int g_ltc_check_count = 0;
static __device__ int g_ltc_check_site = 0;
__device__ __noinline__ static void ltc_check_fail(int site) {
  atomicAdd(&g_ltc_check_count, 1);
  atomicCAS(&g_ltc_check_site, 0, site);
}
#define LTC_CHECK(cond, site) \
  do {                        \
    if (!(cond)) ::ltc::ltc_check_fail(site); \
  } while (0)
// evaluates to true when the access must be skipped
#define LTC_CHECKED_SKIP(cond, site) (!(cond) ? (::ltc::ltc_check_fail(site), true) : false)
static int ltc_check_read(int* count, int* site) {
  int c = 0, s = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&c, g_ltc_check_count, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&s, g_ltc_check_site, sizeof(int));
  const int zero = 0;
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_ltc_check_count, &zero, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_ltc_check_site, &zero, sizeof(int));
  *count += c;
  if (!*site) *site = s;
  return (int)e;
}
static struct LtcCheckRegistration {
  LtcCheckRegistration() { register_check_reader(&ltc_check_read); }
} s_ltc_check_registration;
#else
#define LTC_CHECK(cond, site) ((void)0)
#define LTC_CHECKED_SKIP(cond, site) false
#endif

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed FP32 (Blackwell f32x2): one instruction, two IEEE fp32 results ----
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 tanh2(float2 a) { return make_float2(tanh_approx(a.x), tanh_approx(a.y)); }

// Backward-pass gate with one MUFU op: sigmoid(z) = 0.5 + 0.5*tanh(z/2), given the
// half-scale pack (sh, nh) = (sigma/2, -sigma*mu/2) so that z/2 = sh*v + nh.
// tanh.approx has a relative error of about 2^-11; the adjoint tolerates it
// (gradient bar rtol 5e-2), the forward state does not use it.
__device__ __forceinline__ float gate_tanh(float sh, float nh, float v) {
  return fmaf(0.5f, tanh_approx(fmaf(sh, v, nh)), 0.5f);
}

// ---------------------------------------------------------------------------
// Transposed reduction across the TPC lanes that share one neuron.
//
// Each of the TPC lanes (contiguous lanes, TPC a power of two <= 32) holds SB
// partial sums, one per sample of a block.  Recursive halving exchanges half of
// the remaining samples per step, so that after log2(min(SB,TPC)) exchanges
// every lane holds full sums for SB/TPC samples (or, when TPC > SB, the
// remaining steps are butterflies and TPC/SB lanes hold the same sample).
// Fixed order => bitwise deterministic.
//   NV  : number of independent value arrays reduced with the same pattern
//   out : x[v][0 .. OWN-1] hold the sums for samples own_base() + i
// ---------------------------------------------------------------------------
template <int TPC, int SB>
struct LaneReduce {
  static constexpr int OWN = (SB >= TPC) ? SB / TPC : 1;

  template <int NV>
  __device__ __forceinline__ static void run(float (&x)[NV][SB], int lane) {
    int count = SB;
#pragma unroll
    for (int stride = TPC / 2; stride >= 1; stride >>= 1) {
      const bool hi = (lane & stride) != 0;
      if (count > 1) {
        const int half = count / 2;
#pragma unroll
        for (int k = 0; k < SB / 2; ++k) {
          if (k < half) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
              const float send = hi ? x[v][k] : x[v][k + half];
              const float keep = hi ? x[v][k + half] : x[v][k];
              x[v][k] = keep + __shfl_xor_sync(0xffffffffu, send, stride);
            }
          }
        }
        count = half;
      } else {
#pragma unroll
        for (int v = 0; v < NV; ++v) x[v][0] += __shfl_xor_sync(0xffffffffu, x[v][0], stride);
      }
    }
  }

  // first sample index (within the block) whose sums this lane holds
  __device__ __forceinline__ static int own_base(int lane) {
    int base = 0, count = SB;
#pragma unroll
    for (int stride = TPC / 2; stride >= 1; stride >>= 1) {
      if (count > 1) {
        const int half = count / 2;
        if (lane & stride) base += half;
        count = half;
      }
    }
    return base;
  }

  // true for exactly one lane among those holding identical sums
  __device__ __forceinline__ static bool writer(int lane) {
    int count = SB;
    bool w = true;
#pragma unroll
    for (int stride = TPC / 2; stride >= 1; stride >>= 1) {
      if (count > 1) {
        count /= 2;
      } else if (lane & stride) {
        w = false;
      }
    }
    return w;
  }
};

// 4-byte asynchronous global->shared copy (Ampere+ cp.async, valid on sm_100a)
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
// 4-byte copy that writes 0 instead when !valid (src-size 0: nothing is read)
__device__ __forceinline__ void cp_async4_zfill(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(valid ? 4 : 0));
}
// Rows 0 .. nrows-1 of H floats each (row s at src + s * src_ld) -> shared rows of
// stride ld floats, asynchronously: 16-byte copies when both bases are 16-byte aligned
// and H, src_ld and ld are multiples of 4 (every row then stays aligned), else 4-byte
// copies (a caller's workspace need not be 16-byte aligned).
__device__ __forceinline__ void stage_rows_async(float* dst, int ld, const float* src, long long src_ld,
                                                 int nrows, int H, int tid, int nt) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  if (aligned && ((H | ld | (int)(src_ld & 3)) & 3) == 0) {
    const int h4 = H >> 2;
    for (int i = tid; i < nrows * h4; i += nt) {
      const int s = i / h4, k = i - s * h4;
      cp_async16(dst + s * ld + 4 * k, src + s * src_ld + 4 * k);
    }
  } else {
    for (int i = tid; i < nrows * H; i += nt) {
      const int s = i / H, h = i - s * H;
      cp_async4(dst + s * ld + h, src + s * src_ld + h);
    }
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

}  // namespace ltc
