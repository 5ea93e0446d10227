// Persistent recurrent kernels for any H up to 512 ("wide" path; H > 64 by default).
//
// The synapse matrix no longer fits in one CTA's registers, so the gate pack is
// streamed from L2 through a double-buffered shared-memory chunk of PC rows
// (cp.async), shared by SG sample groups of the CTA.  Each thread owns one
// neuron for NSPT samples:
//   forward : thread = (column q, sample group sg), sums over all presynaptic p
//             itself -- no cross-thread reduction;
//   backward: thread = (row p, sample group sg), sums dL/dv[p] over all q itself;
//             synapse gradients are accumulated in a per-(CTA, sample group)
//             slab in global memory (layout [q][p], coalesced), read-modify-
//             written once per chunk and unfold, amortised over NSPT samples.
// As in the register-resident kernels, one launch covers all T*U unfolds.
#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace ltc {

namespace {

__host__ __device__ inline int wide_pc(int HPW) {
  return HPW <= 128 ? 32 : (HPW <= 256 ? 16 : 8);
}

template <int NSPT>
__global__ void __launch_bounds__(512, 1) rec_fwd_wide(RecFwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int HPW = a.HP;
  const int SG = blockDim.x / HPW;
  const int PC = wide_pc(HPW);
  const int NC = HPW / PC;
  const int ns = SG * NSPT;
  float4* pks = reinterpret_cast<float4*>(smem);     // [2][PC][HPW]
  float* vbuf = smem + 2 * 4 * PC * HPW;              // [2][ns][HPW]
  float* snb = vbuf + 2 * ns * HPW;                   // [2][ns][HPW]
  float* sdb = snb + 2 * ns * HPW;                    // [2][ns][HPW]

  const int tid = threadIdx.x;
  const int q = tid % HPW, sg = tid / HPW;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int b0 = blockIdx.x * ns;
  const int nvalid = min(ns, B - b0);
  const float4 nq = a.nrn[q];
  const float cm = nq.x, cmgl = nq.x + nq.y, glvl = nq.w;

  for (int i = tid; i < 6 * ns * HPW; i += blockDim.x) vbuf[i] = 0.f;
  __syncthreads();
  if (a.h0)
    for (int i = tid; i < nvalid * H; i += blockDim.x)
      vbuf[(i / H) * HPW + (i % H)] = a.h0[(long long)b0 * H + i];

  auto stage_chunk = [&](int c, int buf) {
    float4* dst = pks + buf * PC * HPW;
    const float4* src = a.pack + (long long)c * PC * HPW;
    for (int i = tid; i < PC * HPW; i += blockDim.x) cp_async16(dst + i, src + i);
    cp_async_commit();
  };
  stage_chunk(0, 0);
  int cc = 0;  // running chunk counter (buffer = cc % 2)
  int cur = 0;
  for (int t = 0; t < T; ++t) {
    float* snt = snb + (t & 1) * ns * HPW;
    float* sdt = sdb + (t & 1) * ns * HPW;
    for (int i = tid; i < nvalid * H; i += blockDim.x) {
      const int s = i / H, h = i % H;
      const long long row = (long long)(b0 + s) * T + t;
      snt[s * HPW + h] = a.sn[row * H + h];
      sdt[s * HPW + h] = a.sd[row * H + h];
    }
    for (int u = 0; u < U; ++u) {
      const long long n = (long long)t * U + u;
      const float* vc = vbuf + cur * ns * HPW;
      float* vn = vbuf + (cur ^ 1) * ns * HPW;
      // act = 0.5 + 0.5*tanh(z/2): accumulate sum w*tanh and add sum w at the end
      float accn[NSPT], accd[NSPT], cwe = 0.f, cwp = 0.f;
#pragma unroll
      for (int i = 0; i < NSPT; ++i) accn[i] = accd[i] = 0.f;
      for (int c = 0; c < NC; ++c, ++cc) {
        cp_async_wait_all();
        __syncthreads();
        stage_chunk((c + 1) % NC, (cc + 1) & 1);
        const float4* pk = pks + (cc & 1) * PC * HPW + q;
        const float* vrow = vc + (sg * NSPT) * HPW + c * PC;
        for (int pp = 0; pp < PC; ++pp) {
          const float4 w = pk[pp * HPW];
          cwe += w.w;
          cwp += w.z;
#pragma unroll
          for (int i = 0; i < NSPT; ++i) {
            const float th = tanh_approx(fmaf(w.x, vrow[i * HPW + pp], w.y));
            accn[i] = fmaf(w.w, th, accn[i]);
            accd[i] = fmaf(w.z, th, accd[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < NSPT; ++i) {
        const int s = sg * NSPT + i;
        const float v = vc[s * HPW + q];
        const float num = (cm * v + glvl) + (0.5f * (cwe + accn[i]) + snt[s * HPW + q]);
        const float r = rcp_approx((cmgl + (0.5f * (cwp + accd[i]) + sdt[s * HPW + q])) + a.eps);
        const float vnew = num * r;
        if (q < H && s < nvalid) {
          vn[s * HPW + q] = vnew;
          const long long bs = b0 + s;
          if (a.V) {
            a.V[(n * B + bs) * H + q] = v;
            a.R[(n * B + bs) * H + q] = r;
          }
          if (u == U - 1 && a.out) a.out[(bs * T + t) * H + q] = vnew;
        }
      }
      cur ^= 1;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const float* vc = vbuf + cur * ns * HPW;
  for (int i = tid; i < nvalid * H; i += blockDim.x) {
    const int s = i / H, h = i % H;
    const long long bs = b0 + s;
    if (a.hT) a.hT[bs * H + h] = vc[s * HPW + h];
    if (a.V) a.V[((long long)T * U * B + bs) * H + h] = vc[s * HPW + h];
  }
}

template <int NSPT>
__global__ void __launch_bounds__(512, 1) rec_bwd_wide(RecBwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int HPW = a.HP;
  const int SG = blockDim.x / HPW;
  const int PC = wide_pc(HPW);
  const int NC = HPW / PC;
  const int ns = SG * NSPT;
  float4* pks = reinterpret_cast<float4*>(smem);  // [2][PC][HPW], rows q, columns p
  float* AN = smem + 2 * 4 * PC * HPW;             // [2][ns][HPW]
  float* AD = AN + 2 * ns * HPW;                   // [2][ns][HPW]

  const int tid = threadIdx.x;
  const int p = tid % HPW, sg = tid / HPW;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int b0 = blockIdx.x * ns;
  const int nvalid = min(ns, B - b0);
  const long long NTU = (long long)T * U;
  const long long hp2 = (long long)HPW * HPW;
  float* slab = a.part + ((long long)blockIdx.x * SG + sg) * 4 * hp2 + p;
  const float4 np_ = a.nrn[p];
  const float cm = np_.x, gl = np_.y, vl = np_.z;
  const bool pvalid = p < H;

  for (int i = tid; i < 4 * ns * HPW; i += blockDim.x) AN[i] = 0.f;
  for (int q = 0; q < (a.accumulate ? 0 : HPW); ++q) {  // kept when accumulating segments
    slab[q * HPW] = 0.f;
    slab[hp2 + q * HPW] = 0.f;
    slab[2 * hp2 + q * HPW] = 0.f;
    slab[3 * hp2 + q * HPW] = 0.f;
  }
  float gcm = 0.f, ggl = 0.f, gvl = 0.f;
  float dir[NSPT], gsn[NSPT], gsd[NSPT], vcur[NSPT];
  bool ok[NSPT];
  long long bs[NSPT];
#pragma unroll
  for (int i = 0; i < NSPT; ++i) {
    const int s = sg * NSPT + i;
    ok[i] = pvalid && s < nvalid;
    bs[i] = b0 + s;
    dir[i] = gsn[i] = gsd[i] = vcur[i] = 0.f;
  }
  __syncthreads();

  auto vload = [&](long long m, int i) { return a.V[(m * B + bs[i]) * H + p]; };
  auto rload = [&](long long m, int i) { return a.R[(m * B + bs[i]) * H + p]; };
  // prep of unfold m for own sample i, given g = dL/dv_{m+1}[p] and v_{m+1} = vout
  auto prep = [&](long long m, int i, float gval, float vin, float vout, float r, bool first) {
    const float an = gval * r;
    const float ad = -an * vout;
    gcm = fmaf(an, vin - vout, gcm);
    ggl = fmaf(an, vl - vout, ggl);
    gvl = fmaf(an, gl, gvl);
    gsn[i] = first ? an : gsn[i] + an;
    gsd[i] = first ? ad : gsd[i] + ad;
    dir[i] = an * cm;
    const int idx = (int)(m & 1) * ns * HPW + (sg * NSPT + i) * HPW + p;
    AN[idx] = an;
    AD[idx] = ad;
  };

#pragma unroll
  for (int i = 0; i < NSPT; ++i) {
    if (ok[i]) {
      float gval = a.gout[bs[i] * a.go_sb + (long long)(T - 1) * a.go_st + (long long)p * a.go_sh];
      if (a.gstate) gval += a.gstate[bs[i] * H + p];
      const float vin = vload(NTU - 1, i);
      prep(NTU - 1, i, gval, vin, vload(NTU, i), rload(NTU - 1, i), true);
      vcur[i] = vin;
    }
  }

  auto stage_chunk = [&](int c, int buf) {
    float4* dst = pks + buf * PC * HPW;
    const float4* src = a.packT + (long long)c * PC * HPW;
    for (int i = tid; i < PC * HPW; i += blockDim.x) cp_async16(dst + i, src + i);
    cp_async_commit();
  };
  stage_chunk(0, 0);
  int cc = 0;
  for (long long n = NTU - 1; n >= 0; --n) {
    const int t = (int)(n / U), k = (int)(n % U);
    float vprev[NSPT], rprev[NSPT], dv[NSPT];
#pragma unroll
    for (int i = 0; i < NSPT; ++i) {
      dv[i] = 0.f;
      vprev[i] = (ok[i] && n > 0) ? vload(n - 1, i) : 0.f;
      rprev[i] = (ok[i] && n > 0) ? rload(n - 1, i) : 0.f;
    }
    const float* ans = AN + (int)(n & 1) * ns * HPW + (sg * NSPT) * HPW;
    const float* ads = AD + (int)(n & 1) * ns * HPW + (sg * NSPT) * HPW;
    for (int c = 0; c < NC; ++c, ++cc) {
      cp_async_wait_all();
      __syncthreads();
      stage_chunk((c + 1) % NC, (cc + 1) & 1);
      const float4* pk = pks + (cc & 1) * PC * HPW + p;
      for (int qq = 0; qq < PC; ++qq) {
        const int q = c * PC + qq;
        const float4 w = pk[qq * HPW];
        float* gp = slab + (long long)q * HPW;
        float g0 = gp[0], g1 = gp[hp2], g2 = gp[2 * hp2], g3 = gp[3 * hp2];
#pragma unroll
        for (int i = 0; i < NSPT; ++i) {
          const float an = ans[i * HPW + q];
          const float ad = ads[i * HPW + q];
          const float act = gate_tanh(w.x, w.y, vcur[i]);
          const float sp = fmaf(-act, act, act);
          const float dz = fmaf(an, w.w, ad * w.z) * sp;
          g0 = fmaf(an, act, g0);
          g1 = fmaf(ad, act, g1);
          g2 += dz;
          g3 = fmaf(dz, vcur[i], g3);
          dv[i] = fmaf(dz, w.x, dv[i]);
        }
        gp[0] = g0;
        gp[hp2] = g1;
        gp[2 * hp2] = g2;
        gp[3 * hp2] = g3;
      }
    }
#pragma unroll
    for (int i = 0; i < NSPT; ++i) {
      if (!ok[i]) continue;
      float gval = fmaf(2.0f, dv[i], dir[i]);
      if (k == 0) {
        const long long row = bs[i] * T + t;
        a.gsn[row * H + p] = gsn[i];
        a.gsd[row * H + p] = gsd[i];
        if (t == 0) {
          a.gh0[bs[i] * H + p] = gval;
          continue;
        }
        gval += a.gout[bs[i] * a.go_sb + (long long)(t - 1) * a.go_st + (long long)p * a.go_sh];
      }
      prep(n - 1, i, gval, vprev[i], vcur[i], rprev[i], k == 0);
      vcur[i] = vprev[i];
    }
  }
  cp_async_wait_all();
  float* pn = a.partn + ((long long)blockIdx.x * SG + sg) * 3 * HPW;
  pn[p] = a.accumulate ? pn[p] + gcm : gcm;
  pn[HPW + p] = a.accumulate ? pn[HPW + p] + ggl : ggl;
  pn[2 * HPW + p] = a.accumulate ? pn[2 * HPW + p] + gvl : gvl;
}

template <int NSPT>
cudaError_t go_fwd(const RecFwdArgs& a, const RecPlan& pl, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(rec_fwd_wide<NSPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)pl.smem_fwd);
  if (e != cudaSuccess) return e;
  rec_fwd_wide<NSPT><<<pl.grid_fwd, pl.threads_fwd, pl.smem_fwd, st>>>(a);
  return cudaGetLastError();
}

template <int NSPT>
cudaError_t go_bwd(const RecBwdArgs& a, const RecPlan& pl, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(rec_bwd_wide<NSPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)pl.smem_bwd);
  if (e != cudaSuccess) return e;
  rec_bwd_wide<NSPT><<<pl.grid_bwd, pl.threads_bwd, pl.smem_bwd, st>>>(a);
  return cudaGetLastError();
}

int nspt_of(int ns, int SG) { return ns / SG; }

}  // namespace

void plan_wide(RecPlan& p, int B, int H, int num_sms) {
  const int HPW = round_up(H, 32);
  p.HP = HPW;
  const int SG = HPW >= 512 ? 1 : 512 / HPW;
  const int PC = wide_pc(HPW);
  const size_t smem_cap = 220 * 1024;
  // samples per thread: minimise waves x samples-per-thread (time), ties -> fewer CTAs
  int best = 1;
  long long best_cost = -1;
  for (int nspt = 1; nspt <= 8; nspt *= 2) {
    const int ns = SG * nspt;
    const size_t sf = (size_t)2 * PC * HPW * 16 + (size_t)6 * ns * HPW * 4;
    const size_t sb = (size_t)2 * PC * HPW * 16 + (size_t)4 * ns * HPW * 4;
    if (sf > smem_cap || sb > smem_cap) break;
    const long long grid = (B + ns - 1) / ns;
    const long long cost = ((grid + num_sms - 1) / num_sms) * nspt;
    if (best_cost < 0 || cost <= best_cost) {
      best_cost = cost;
      best = nspt;
    }
  }
  p.ns_fwd = p.ns_bwd = SG * best;
  p.grid_fwd = p.grid_bwd = (B + p.ns_fwd - 1) / p.ns_fwd;
  p.threads_fwd = p.threads_bwd = HPW * SG;
  p.slots_bwd = p.grid_bwd * SG;
  p.smem_fwd = (size_t)2 * PC * HPW * 16 + (size_t)6 * p.ns_fwd * HPW * 4;
  p.smem_bwd = (size_t)2 * PC * HPW * 16 + (size_t)4 * p.ns_bwd * HPW * 4;
}

cudaError_t launch_wide_fwd(const RecFwdArgs& a, const RecPlan& pl, cudaStream_t st) {
  switch (nspt_of(pl.ns_fwd, pl.threads_fwd / pl.HP)) {
    case 1: return go_fwd<1>(a, pl, st);
    case 2: return go_fwd<2>(a, pl, st);
    case 4: return go_fwd<4>(a, pl, st);
    default: return go_fwd<8>(a, pl, st);
  }
}

cudaError_t launch_wide_bwd(const RecBwdArgs& a, const RecPlan& pl, cudaStream_t st) {
  switch (nspt_of(pl.ns_bwd, pl.threads_bwd / pl.HP)) {
    case 1: return go_bwd<1>(a, pl, st);
    case 2: return go_bwd<2>(a, pl, st);
    case 4: return go_bwd<4>(a, pl, st);
    default: return go_bwd<8>(a, pl, st);
  }
}

}  // namespace ltc
