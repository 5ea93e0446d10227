// Persistent recurrent kernels for H <= 64 (padded to HP = 32 or 64).
//
// One CTA owns a group of `ns` samples for the whole sequence (all T*U
// unfolds in one launch) and keeps every recurrent synapse of the cell in
// registers: each thread holds RPT x 8 synapses (RPT = 2 at HP = 64: 256
// threads x 16 synapses), 4 gate-pack values per synapse and, in the backward
// kernel, 4 gradient accumulators per synapse.  Per unfold the only traffic is
// the sample state in shared memory; one __syncthreads() separates unfolds
// (Jacobi update: every new v is computed from the previous unfold's v,
// double-buffered -- unlike an in-place update).
//
// Forward thread map:  lane group g = tid % TPC (TPC = HP/8 lanes), column group
//   c = tid / TPC owns the RPT columns q_r = c + r*HP/RPT and presynaptic rows
//   p(j) = (j/4)*(HP/2) + 4g + j%4 (j < 8).  The 8 operand loads per sample are
//   shared by the RPT columns.
// Backward thread map: row group c owns rows p_r = c + r*HP/RPT and columns q(j).
// The interleaved p(j)/q(j) make the float4 shared-memory loads bank-conflict
// free.  Per block of kSB samples, RPT*kSB partial sums are reduced across the
// TPC lanes by a transposed (recursive-halving) reduction after which every lane
// owns one (neuron, sample) item and runs its per-neuron "tail".
#include <cooperative_groups.h>

#include <mutex>

#include "ltc_cluster.cuh"
#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace cg = cooperative_groups;

namespace ltc {

// bounded cluster waits that expired (see ltc_cluster.cuh)
__device__ int g_ltc_wait_timeouts = 0;

namespace {

constexpr int kSB = 4;  // samples per register block
constexpr int kMaxBlk = 8;  // sample blocks per group of a cluster kernel (CL > 1)

// Neurons per thread and resident CTAs per SM of each kernel at HP = 64 (tuned on B200).
#ifndef LTC_FWD_RPT
#define LTC_FWD_RPT 1
#endif
#ifndef LTC_FWD_CTAS
#define LTC_FWD_CTAS 1
#endif
#ifndef LTC_BWD_RPT
#define LTC_BWD_RPT 2
#endif
#ifndef LTC_BWD_RPT128
#define LTC_BWD_RPT128 2
#endif

template <int HP, int RPT_, int CL>
struct Geometry {
  static constexpr int RPT = RPT_;              // neurons (rows / columns) per thread
  static constexpr int TPC = HP / 8;            // lanes sharing a neuron group
  static constexpr int NEUR = HP / CL;          // neurons owned by one CTA of the cluster
  static constexpr int NG = NEUR / RPT;         // neuron groups
  static constexpr int NT = NG * TPC;           // threads
  static constexpr int NI = RPT * kSB;          // reduced items per block
  static constexpr int LDV = HP + 4;            // padded row stride of per-sample vectors
  __device__ __forceinline__ static int sub(int j, int g) { return (j / 4) * (HP / 2) + 4 * g + (j % 4); }
};


// Cluster helpers: with CL > 1 the CTAs of a cluster share one sample group and
// each owns HP/CL neurons; per-neuron results of an unfold are sent to every
// CTA's shared memory with st.async and awaited on a per-slot mbarrier
// (ltc_cluster.cuh); the hardware cluster barrier runs only at start and end.
template <int CL>
__device__ __forceinline__ void group_sync() {
  if constexpr (CL > 1) cg::this_cluster().sync();
  else __syncthreads();
}
template <int CL>
__device__ __forceinline__ int group_rank() {
  if constexpr (CL > 1) return (int)cg::this_cluster().block_rank();
  else return 0;
}
template <int HP>
constexpr int cluster_of() { return HP > 64 ? 4 : 1; }

template <int HP>
constexpr int fwd_rpt() { return HP >= 64 ? LTC_FWD_RPT : 1; }
template <int HP>
constexpr int fwd_ctas() { return HP >= 64 ? LTC_FWD_CTAS : 1; }
template <int HP>
constexpr int bwd_rpt() { return HP >= 128 ? LTC_BWD_RPT128 : HP >= 64 ? LTC_BWD_RPT : 1; }

template <int HP>
__global__ void __launch_bounds__(Geometry<HP, fwd_rpt<HP>(), cluster_of<HP>()>::NT, fwd_ctas<HP>())
    rec_fwd_fast(RecFwdArgs a) {
  constexpr int CL = cluster_of<HP>();
  using G = Geometry<HP, fwd_rpt<HP>(), CL>;
  constexpr int TPC = G::TPC, NT = G::NT, LDV = G::LDV, RPT = G::RPT, NG = G::NG;
  using LR = LaneReduce<TPC, G::NI>;
  extern __shared__ __align__(16) float smem[];
  const int ns = a.ns;
  float* vbuf = smem;                // [2][ns][LDV]
  float* snb2 = vbuf + 2 * ns * LDV;  // [2][ns][LDV]: step t in slot t & 1
  float* sdb2 = snb2 + 2 * ns * LDV;  // [2][ns][LDV]

  const int tid = threadIdx.x, lane = tid & 31;
  const int nb = group_rank<CL>() * G::NEUR;  // first neuron of this CTA
  const int c = nb + tid / TPC, g = tid % TPC;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int b0 = (blockIdx.x / CL) * ns;
  const int nvalid = min(ns, B - b0);
  const int nblk = (nvalid + kSB - 1) / kSB;

  float sl[RPT][8], nm[RPT][8], wp[RPT][8], we[RPT][8];
#pragma unroll
  for (int r = 0; r < RPT; ++r)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 pk = a.pack[G::sub(j, g) * HP + c + r * NG];
      sl[r][j] = pk.x; nm[r][j] = pk.y; wp[r][j] = pk.z; we[r][j] = pk.w;
    }
  float cwe[RPT], cwp[RPT];
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    cwe[r] = cwp[r] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      we[r][j] *= 0.5f;
      wp[r][j] *= 0.5f;
      cwe[r] += we[r][j];
      cwp[r] += wp[r][j];
    }
  }
  float2 sl2[RPT][4], nm2[RPT][4], wp2[RPT][4], we2[RPT][4];
#pragma unroll
  for (int r = 0; r < RPT; ++r)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sl2[r][k] = make_float2(sl[r][2 * k], sl[r][2 * k + 1]);
      nm2[r][k] = make_float2(nm[r][2 * k], nm[r][2 * k + 1]);
      wp2[r][k] = make_float2(wp[r][2 * k], wp[r][2 * k + 1]);
      we2[r][k] = make_float2(we[r][2 * k], we[r][2 * k + 1]);
    }
  // the one (column, sample-in-block) item this lane finishes
  const int own = LR::own_base(lane);
  const int orow = own / kSB, osmp = own % kSB;
  const int q = c + orow * NG;
  const float4 nq = a.nrn[q];
  const float cm = nq.x, cmgl = nq.x + nq.y, glvl = nq.w;
  const bool qvalid = q < H;
  const bool writer = LR::writer(lane);

  // vbuf arrivals (CL > 1): one mbarrier per (slot, sample block), so that a
  // block's pass starts as soon as that block's values are in, while the
  // exchange of the other blocks is still in flight
  __shared__ __align__(8) uint64_t xbar[2][kMaxBlk];
  __shared__ int xabort;
  const uint32_t xbytes = (uint32_t)(HP * kSB * sizeof(float));  // per block and phase
  if constexpr (CL > 1) {
    if (tid == 0) {
      xabort = 0;
      for (int i = 0; i < 2 * nblk; ++i) mbar_init(smem_addr(&xbar[i & 1][i >> 1]), 1);
      mbar_init_fence();
      for (int i = 0; i < 2 * nblk; ++i) mbar_arm(smem_addr(&xbar[i & 1][i >> 1]), xbytes);
    }
  }
  uint32_t xphase = 0;  // parity bit per slot
  for (int i = tid; i < 6 * ns * LDV; i += NT) smem[i] = 0.f;
  __syncthreads();
  if (a.h0) {
    for (int i = tid; i < nvalid * H; i += NT) {
      const int s = i / H, h = i % H;
      vbuf[s * LDV + h] = a.h0[(long long)(b0 + s) * H + h];
    }
  }
  // the sensory sums of step t + 1 are copied in (cp.async) while step t unfolds
  auto stage_sens = [&](int t) {
    float* dn = snb2 + (t & 1) * ns * LDV;
    float* dd = sdb2 + (t & 1) * ns * LDV;
    const long long row0 = (long long)b0 * T + t;  // sample s's row is row0 + s * T
    stage_rows_async(dn, LDV, a.sn + row0 * H, (long long)T * H, nvalid, H, tid, NT);
    stage_rows_async(dd, LDV, a.sd + row0 * H, (long long)T * H, nvalid, H, tid, NT);
    cp_async_commit();
  };
  stage_sens(0);
  cp_async_wait_all();
  group_sync<CL>();  // every CTA of the group initialised before any remote store
  int cur = 0;
  for (int t = 0; t < T; ++t) {
    __syncthreads();  // step t's sums visible; slot (t + 1) & 1 no longer read
    if (t + 1 < T) stage_sens(t + 1);
    const float* __restrict__ snb = snb2 + (t & 1) * ns * LDV;
    const float* __restrict__ sdb = sdb2 + (t & 1) * ns * LDV;
    for (int u = 0; u < U; ++u) {
      const long long n = (long long)t * U + u;
      const float* __restrict__ vc = vbuf + cur * ns * LDV;
      float* __restrict__ vn = vbuf + (cur ^ 1) * ns * LDV;
      for (int blk = 0; blk < nblk; ++blk) {
        if constexpr (CL > 1) {  // this block's v of unfold n, from every CTA of the group
          if (n > 0) {
            const uint32_t bar = smem_addr(&xbar[cur][blk]);
            mbar_wait(bar, (xphase >> cur) & 1u, &xabort, &g_ltc_wait_timeouts);
            if (tid == 0 && n + 1 < (long long)T * U) mbar_arm(bar, xbytes);
          }
        }
        float acc[2][G::NI];
#pragma unroll
        for (int i = 0; i < kSB; ++i) {
          const float* vr = vc + (blk * kSB + i) * LDV + 4 * g;
          const float4 va = *reinterpret_cast<const float4*>(vr);
          const float4 vb = *reinterpret_cast<const float4*>(vr + HP / 2);
          const float v8[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
          for (int r = 0; r < RPT; ++r) {
            // act = 0.5 + 0.5*tanh(z/2): the constant halves are folded into
            // cwe/cwp, the weights into the half-scale registers; synapses j and
            // j+1 run as one packed f32x2 lane pair.
            float2 sn2 = make_float2(cwe[r], 0.f), sd2 = make_float2(cwp[r], 0.f);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 vv = make_float2(v8[2 * k], v8[2 * k + 1]);
              const float2 th = tanh2(fma2(sl2[r][k], vv, nm2[r][k]));
              sn2 = fma2(we2[r][k], th, sn2);
              sd2 = fma2(wp2[r][k], th, sd2);
            }
            const float sn_ = sn2.x + sn2.y, sd_ = sd2.x + sd2.y;
            acc[0][r * kSB + i] = sn_;
            acc[1][r * kSB + i] = sd_;
          }
        }
        LR::template run<2>(acc, lane);
        const int s = blk * kSB + osmp;
        LTC_CHECK(s < ns && q >= 0 && q < HP, 401);
        const float v = vc[s * LDV + q];
        const float wn = acc[0][0] + snb[s * LDV + q];
        const float wd = acc[1][0] + sdb[s * LDV + q];
        const float num = (cm * v + glvl) + wn;
        const float rr = rcp_approx((cmgl + wd) + a.eps);
        const float vnew = num * rr;
        const bool ok = qvalid && s < nvalid;
        if constexpr (CL > 1) {
          // every item of the group is sent (zeros for padding): the phase byte count
          if (writer) st_async_all<CL>(vn + s * LDV + q, ok ? vnew : 0.f, smem_addr(&xbar[cur ^ 1][blk]));
        } else {
          if (writer && ok) vn[s * LDV + q] = vnew;
        }
        if (writer && ok) {
          const long long bs = b0 + s;
          if (a.V) {
            a.V[(n * B + bs) * H + q] = v;
            a.R[(n * B + bs) * H + q] = rr;
          }
          if (u == U - 1 && a.out) a.out[(bs * T + t) * H + q] = vnew;
        }
      }
      if constexpr (CL > 1) {
        if (n > 0) xphase ^= 1u << cur;
      } else {
        __syncthreads();
      }
      cur ^= 1;
    }
    cp_async_wait_all();
  }
  if constexpr (CL > 1) {  // the last unfold's v from every CTA of the group
    for (int blk = 0; blk < nblk; ++blk)
      mbar_wait(smem_addr(&xbar[cur][blk]), (xphase >> cur) & 1u, &xabort, &g_ltc_wait_timeouts);
  }
  const float* vc = vbuf + cur * ns * LDV;
  for (int i = tid; i < nvalid * G::NEUR; i += NT) {
    const int s = i / G::NEUR, h = nb + i % G::NEUR;
    if (h >= H) continue;
    const long long bs = b0 + s;
    if (a.hT) a.hT[bs * H + h] = vc[s * LDV + h];
    if (a.V) a.V[((long long)T * U * B + bs) * H + h] = vc[s * LDV + h];
  }
  if constexpr (CL > 1) cg::this_cluster().sync();  // no CTA leaves while a peer may address it
}

// Backward: reverse sweep over n = T*U-1 .. 0 with the adjoint of each unfold.
//  AN/AD[s][q]   = a_n = g*r, a_d = -g*v'*r of the unfold being processed
//  VS[n%3][s][.] = saved V[n] (3 buffers: current, next, prefetch)
//  RS[n%2][s][.] = saved R[n]
//  DIR[s][p]     = direct term g*cm*r of the unfold being processed
//  GSN/GSD[s][p] = running sums of a_n / a_d over the unfolds of the current step
template <int HP>
__global__ void __launch_bounds__(Geometry<HP, bwd_rpt<HP>(), cluster_of<HP>()>::NT, 1)
    rec_bwd_fast(RecBwdArgs a) {
  constexpr int CL = cluster_of<HP>();
  using G = Geometry<HP, bwd_rpt<HP>(), CL>;
  constexpr int TPC = G::TPC, NT = G::NT, LDV = G::LDV, RPT = G::RPT, NG = G::NG;
  using LR = LaneReduce<TPC, G::NI>;
  extern __shared__ __align__(16) float smem[];
  const int ns = a.ns;
  const int SL = ns * LDV;  // one per-sample slab
  float* AN = smem;          // [2]
  float* AD = AN + 2 * SL;   // [2]
  float* VS = AD + 2 * SL;   // [3]
  float* RS = VS + 3 * SL;   // [2]
  float* DIR = RS + 2 * SL;
  float* GSN = DIR + SL;
  float* GSD = GSN + SL;
  float* GO = GSD + SL;      // [2]: 15 slabs, then [5][HP][TPC] for the final per-neuron sums
  float* red = GO + 2 * SL;

  const int tid = threadIdx.x, lane = tid & 31;
  const int nb = group_rank<CL>() * G::NEUR;  // first row of this CTA
  const int c = nb + tid / TPC, g = tid % TPC;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int grp = blockIdx.x / CL;
  const int b0 = grp * ns;
  const int nvalid = min(ns, B - b0);
  const int nblk = (nvalid + kSB - 1) / kSB;
  const int NTU = T * U;  // unfolds in the sequence

  // synapses j = 2k, 2k+1 of a row are one packed f32x2 pair
  float2 sl2[RPT][4], nm2[RPT][4], wp2[RPT][4], we2[RPT][4];
  float2 Gwe[RPT][4], Gwp[RPT][4], Gdz[RPT][4], Gdzv[RPT][4];
#pragma unroll
  for (int r = 0; r < RPT; ++r)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 p0 = a.pack[(c + r * NG) * HP + G::sub(2 * k, g)];
      const float4 p1 = a.pack[(c + r * NG) * HP + G::sub(2 * k + 1, g)];
      // negated half-scale constants: the gate argument is -z/2, so tanh gives -t
      sl2[r][k] = make_float2(-p0.x, -p1.x);
      nm2[r][k] = make_float2(-p0.y, -p1.y);
      wp2[r][k] = make_float2(p0.z, p1.z);
      we2[r][k] = make_float2(p0.w, p1.w);
      Gwe[r][k] = Gwp[r][k] = Gdz[r][k] = Gdzv[r][k] = make_float2(0.f, 0.f);
    }
  const float2 m1 = make_float2(-1.f, -1.f);
  // the one (row, sample-in-block) item this lane finishes
  const int own = LR::own_base(lane);
  const int orow = own / kSB, osmp = own % kSB;
  const int p = c + orow * NG;
  const float4 np_ = a.nrn[p];
  const float cm = np_.x, gl = np_.y, vl = np_.z;
  const bool pvalid = p < H;
  const bool writer = LR::writer(lane);
  float gcm = 0.f, ggl = 0.f, gvl = 0.f, san = 0.f, sad = 0.f;

  // AN/AD arrivals (CL > 1): one mbarrier per (slot, sample block), so that a
  // block's pass starts as soon as that block's values are in, while the
  // exchange of the other blocks is still in flight
  __shared__ __align__(8) uint64_t xbar[2][kMaxBlk];
  __shared__ int xabort;
  const uint32_t xbytes = (uint32_t)(2 * HP * kSB * sizeof(float));  // per block and phase
  if constexpr (CL > 1) {
    if (tid == 0) {
      xabort = 0;
      for (int i = 0; i < 2 * nblk; ++i) mbar_init(smem_addr(&xbar[i & 1][i >> 1]), 1);
      mbar_init_fence();
      for (int i = 0; i < 2 * nblk; ++i) mbar_arm(smem_addr(&xbar[i & 1][i >> 1]), xbytes);
    }
  }
  uint32_t xphase = 0;  // parity bit per slot
  for (int i = tid; i < 15 * SL; i += NT) smem[i] = 0.f;
  __syncthreads();

  // stage saved slices: V[m] -> VS[m%3], R[m] -> RS[m%2]
  auto stage_v = [&](int m) {
    float* dst = VS + (m % 3) * SL;
    const float* src = a.V + ((long long)m * B + b0) * H;
    stage_rows_async(dst, LDV, src, H, nvalid, H, tid, NT);
  };
  auto stage_r = [&](int m) {
    float* dst = RS + (m % 2) * SL;
    const float* src = a.R + ((long long)m * B + b0) * H;
    stage_rows_async(dst, LDV, src, H, nvalid, H, tid, NT);
  };
  // dL/dout of step tt (strided) -> GO[tt & 1], copied in while later unfolds run;
  // a gradient broadcast over samples and steps (stride 0, e.g. a sum loss) is
  // read in place: it is H values that stay in cache
  const bool go_bcast = a.go_sb == 0 && a.go_st == 0;
  auto stage_go = [&](int tt) {
    if (go_bcast) return;
    float* dst = GO + (tt & 1) * SL;
    for (int i = tid; i < nvalid * H; i += NT) {
      const int s = i / H, h = i % H;
      cp_async4(dst + s * LDV + h, a.gout + (long long)(b0 + s) * a.go_sb + (long long)tt * a.go_st +
                                       (long long)h * a.go_sh);
    }
  };
  stage_v(NTU);
  stage_v(NTU - 1);
  stage_r(NTU - 1);
  if (NTU >= 2) {
    stage_v(NTU - 2);
    stage_r(NTU - 2);
  }
  if (T >= 2) stage_go(T - 2);
  cp_async_commit();
  cp_async_wait_all();
  group_sync<CL>();  // every CTA of the group initialised before any remote store

  // Per-neuron prep of unfold m for (sample s, neuron p) given g = dL/dv_{m+1}[p]:
  // rs/vin/vout/an/ad point at the slabs of R[m], V[m], V[m+1] and the adjoint
  // slabs of unfold m (slot arithmetic done once per unfold by the caller).
  auto prep = [&](const float* rs, const float* vin_s, const float* vout_s, float* an_d, float* ad_d, int s,
                  float gval, bool first_of_step) {
    const int idx = s * LDV + p;
    const float r = rs[idx];
    const float vin = vin_s[idx];
    const float vout = vout_s[idx];
    const float an = gval * r;
    const float ad = -an * vout;
    gcm = fmaf(an, vin - vout, gcm);
    ggl = fmaf(an, vl - vout, ggl);
    gvl = fmaf(an, gl, gvl);
    san += an;
    sad += ad;
    GSN[idx] = first_of_step ? an : GSN[idx] + an;
    GSD[idx] = first_of_step ? ad : GSD[idx] + ad;
    DIR[idx] = an * cm;
    // the synapse pass works in tanh space: it reads a' = -a/4 (see the pass)
    if constexpr (CL > 1) {
      const uint32_t bar = smem_addr(&xbar[(an_d - AN) / SL][s / kSB]);
      st_async_all<CL>(an_d + idx, -0.25f * an, bar);
      st_async_all<CL>(ad_d + idx, -0.25f * ad, bar);
    } else {
      an_d[idx] = -0.25f * an;
      ad_d[idx] = -0.25f * ad;
    }
  };
  // CL > 1: a padding item (row >= H or sample >= nvalid) still completes its bytes
  auto send_zero = [&](float* an_d, float* ad_d, int s) {
    if constexpr (CL > 1) {
      const int idx = s * LDV + p;
      const uint32_t bar = smem_addr(&xbar[(an_d - AN) / SL][s / kSB]);
      st_async_all<CL>(an_d + idx, 0.f, bar);
      st_async_all<CL>(ad_d + idx, 0.f, bar);
    }
  };

  // initial prep of unfold NTU-1: g = dL/dout[:, T-1] + dL/dstate
  if (writer) {
    const int m = NTU - 1;
    for (int blk = 0; blk < nblk; ++blk) {
      const int s = blk * kSB + osmp;
      LTC_CHECK(s < ns && p >= 0 && p < HP, 402);
      if (pvalid && s < nvalid) {
        const long long bs = b0 + s;
        float gval = a.gout[bs * a.go_sb + (long long)(T - 1) * a.go_st + (long long)p * a.go_sh];
        if (a.gstate) gval += a.gstate[bs * H + p];
        prep(RS + (m % 2) * SL, VS + (m % 3) * SL, VS + ((m + 1) % 3) * SL, AN + (m % 2) * SL,
             AD + (m % 2) * SL, s, gval, true);
      } else {
        send_zero(AN + (m % 2) * SL, AD + (m % 2) * SL, s);
      }
    }
  }
  if constexpr (CL == 1) __syncthreads();

  int t = T - 1, k = U - 1;  // n = t*U + k
  for (int n = NTU - 1; n >= 0; --n) {
    // Tails of iteration m read V[m-1], V[m] and R[m-1]; prefetch what the tails
    // of the next iteration (n-1) need beyond that: V[n-2] and R[n-2].  Their
    // slots ((n+1)%3 and n%2) are not read in this iteration.
    if (n >= 2) {
      stage_v(n - 2);
      stage_r(n - 2);
    }
    if (k == 0 && t >= 2) stage_go(t - 2);  // read at step t - 1's last unfold, >= 1 unfold later
    cp_async_commit();

    const int c2 = n % 2, c2m = c2 ^ 1;          // slots of unfold n and n-1 (mod 2)
    const int c3 = n % 3, c3m = (n + 2) % 3;     // slots of V[n] and V[n-1] (mod 3)
    const float* an_s = AN + c2 * SL;
    const float* ad_s = AD + c2 * SL;
    const float* vsn = VS + c3 * SL;
    const float* vsm = VS + c3m * SL;
    const float* rsm = RS + c2m * SL;
    float* an_m = AN + c2m * SL;
    float* ad_m = AD + c2m * SL;
    for (int blk = 0; blk < nblk; ++blk) {
      if constexpr (CL > 1) {  // this block's adjoints of unfold n, from every CTA of the group
        const uint32_t bar = smem_addr(&xbar[c2][blk]);
        mbar_wait(bar, (xphase >> c2) & 1u, &xabort, &g_ltc_wait_timeouts);
        if (tid == 0 && n >= 2) mbar_arm(bar, xbytes);
      }
      float acc[1][G::NI];
#pragma unroll
      for (int i = 0; i < kSB; ++i) {
        const int s = blk * kSB + i;
        const float* ar = an_s + s * LDV + 4 * g;
        const float* dr = ad_s + s * LDV + 4 * g;
        const float4 a0 = *reinterpret_cast<const float4*>(ar);
        const float4 a1 = *reinterpret_cast<const float4*>(ar + HP / 2);
        const float4 d0 = *reinterpret_cast<const float4*>(dr);
        const float4 d1 = *reinterpret_cast<const float4*>(dr + HP / 2);
        const float2 an2[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                               make_float2(a1.z, a1.w)};
        const float2 ad2[4] = {make_float2(d0.x, d0.y), make_float2(d0.z, d0.w), make_float2(d1.x, d1.y),
                               make_float2(d1.z, d1.w)};
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
          const float vp = vsn[s * LDV + c + r * NG];
          const float2 vp2 = make_float2(vp, vp);
          float2 dv = make_float2(0.f, 0.f);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // Tanh space: with tn = tanh(-z/2) = -t and the stored a' = -a/4,
            //   dL/dz = (a_n w_erev + a_d w_pos) act(1-act) = (a'_n w_erev + a'_d w_pos)(tn^2 - 1)
            //   a act  = a/2 + 2 a' tn   (the a/2 part is summed per column by the tails)
            const float2 tn = tanh2(fma2(sl2[r][k], vp2, nm2[r][k]));
            const float2 dz = mul2(fma2(an2[k], we2[r][k], mul2(ad2[k], wp2[r][k])), fma2(tn, tn, m1));
            Gwe[r][k] = fma2(an2[k], tn, Gwe[r][k]);
            Gwp[r][k] = fma2(ad2[k], tn, Gwp[r][k]);
            Gdz[r][k] = add2(Gdz[r][k], dz);
            Gdzv[r][k] = fma2(dz, vp2, Gdzv[r][k]);
            dv = fma2(dz, sl2[r][k], dv);
          }
          acc[0][r * kSB + i] = dv.x + dv.y;
        }
      }
      LR::template run<1>(acc, lane);
      const int s = blk * kSB + osmp;
      LTC_CHECK(s < ns && p >= 0 && p < HP, 403);
      if (writer && !(pvalid && s < nvalid) && n > 0) send_zero(an_m, ad_m, s);
      if (pvalid && writer && s < nvalid) {
        const int idx = s * LDV + p;
        float gval = fmaf(-2.0f, acc[0][0], DIR[idx]);  // dL/dv_n[p] (sl holds -sigma/2)
        const long long bs = b0 + s;
        bool done = false;
        if (k == 0) {
          const long long row = bs * T + t;
          a.gsn[row * H + p] = GSN[idx];
          a.gsd[row * H + p] = GSD[idx];
          if (t == 0) {
            a.gh0[bs * H + p] = gval;
            done = true;
          } else {
            gval += go_bcast ? a.gout[(long long)p * a.go_sh] : GO[((t - 1) & 1) * SL + idx];
          }
        }
        if (!done) prep(rsm, vsm, vsn, an_m, ad_m, s, gval, k == 0);
      }
    }
    if constexpr (CL > 1) xphase ^= 1u << c2;
    cp_async_wait_all();
    __syncthreads();  // staged V/R visible to the whole CTA
    if (--k < 0) {
      k = U - 1;
      --t;
    }
  }

  // partial gradients of this CTA
  float* part = a.part + (long long)grp * 4 * HP * HP;  // rows of the CTAs of a group are disjoint
#pragma unroll
  for (int r = 0; r < RPT; ++r)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int idx = (c + r * NG) * HP + G::sub(j, g);
      const int k = j / 2;
      const bool hi = j & 1;
      const float v0 = hi ? Gwe[r][k].y : Gwe[r][k].x, v1 = hi ? Gwp[r][k].y : Gwp[r][k].x;
      const float v2 = hi ? Gdz[r][k].y : Gdz[r][k].x, v3 = hi ? Gdzv[r][k].y : Gdzv[r][k].x;
      if (a.accumulate) {
        part[idx] += v0;
        part[HP * HP + idx] += v1;
        part[2 * HP * HP + idx] += v2;
        part[3 * HP * HP + idx] += v3;
      } else {
        part[idx] = v0;
        part[HP * HP + idx] = v1;
        part[2 * HP * HP + idx] = v2;
        part[3 * HP * HP + idx] = v3;
      }
    }
  // per-neuron sums: each lane holds the partial of its own row; fixed-order sum
  // over the lanes of the group through shared memory.
  for (int i = tid; i < 5 * HP * TPC; i += NT) red[i] = 0.f;
  __syncthreads();
  if (writer) {
    red[(0 * HP + p) * TPC + g] = gcm;
    red[(1 * HP + p) * TPC + g] = ggl;
    red[(2 * HP + p) * TPC + g] = gvl;
    red[(3 * HP + p) * TPC + g] = san;
    red[(4 * HP + p) * TPC + g] = sad;
  }
  __syncthreads();
  if (tid < G::NEUR) {
    const int row = nb + tid;
    float* pn = a.partn + (long long)grp * 5 * HP;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      float sum = 0.f;
      for (int l = 0; l < TPC; ++l) sum += red[(k * HP + row) * TPC + l];
      pn[k * HP + row] = a.accumulate ? pn[k * HP + row] + sum : sum;
    }
  }
  if constexpr (CL > 1) cg::this_cluster().sync();  // no CTA leaves while a peer may address it
}

template <int CL, typename Args>
cudaError_t launch_grouped(void (*kernel)(Args), const Args& a, int grid, int threads, size_t smem,
                           cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if constexpr (CL == 1) {
    kernel<<<grid, threads, smem, st>>>(a);
    return cudaGetLastError();
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
  }
}

// Host-side bounds checks of a launch's sample grouping against the shared-memory
// layout the kernels index (slabs of ns * LDV floats; sample s < ns; blocks of kSB;
// at most kMaxBlk blocks per group with the cluster exchange): a plan that breaks
// them is refused before any launch.
template <int HP>
bool grouping_ok(int B, int ns, int grid, size_t smem, size_t need_floats) {
  const int CL = cluster_of<HP>();
  return ns > 0 && ns % kSB == 0 && (long long)(grid / CL) * ns >= B && grid % CL == 0 &&
         (CL == 1 || ns / kSB <= kMaxBlk) && smem >= need_floats * sizeof(float) && smem <= 227 * 1024;
}

template <int HP>
cudaError_t launch_fast_fwd(const RecFwdArgs& a, const RecPlan& pl, cudaStream_t st) {
  if (!grouping_ok<HP>(a.B, a.ns, pl.grid_fwd, pl.smem_fwd, (size_t)6 * a.ns * (HP + 4)))
    return cudaErrorInvalidValue;
  return launch_grouped<cluster_of<HP>()>(rec_fwd_fast<HP>, a, pl.grid_fwd,
                                          Geometry<HP, fwd_rpt<HP>(), cluster_of<HP>()>::NT, pl.smem_fwd, st);
}

template <int HP>
cudaError_t launch_fast_bwd(const RecBwdArgs& a, const RecPlan& pl, cudaStream_t st) {
  if (!grouping_ok<HP>(a.B, a.ns, pl.grid_bwd, pl.smem_bwd,
                       (size_t)15 * a.ns * (HP + 4) + 5 * HP * (HP / 8)))
    return cudaErrorInvalidValue;
  return launch_grouped<cluster_of<HP>()>(rec_bwd_fast<HP>, a, pl.grid_bwd,
                                          Geometry<HP, bwd_rpt<HP>(), cluster_of<HP>()>::NT, pl.smem_bwd, st);
}

}  // namespace

// wide-H kernels (ltc_recurrent_wide.cu)
cudaError_t launch_wide_fwd(const RecFwdArgs& a, const RecPlan& p, cudaStream_t st);
cudaError_t launch_wide_bwd(const RecBwdArgs& a, const RecPlan& p, cudaStream_t st);
void plan_wide(RecPlan& p, int B, int H, int num_sms);
// cluster-streamed kernels (ltc_recurrent_stream.cu)
cudaError_t launch_stream_fwd(const RecFwdArgs& a, const RecPlan& p, cudaStream_t st);
cudaError_t launch_stream_bwd(const RecBwdArgs& a, const RecPlan& p, cudaStream_t st);
void plan_stream(RecPlan& p, int B, int H, int num_sms);

namespace {
__global__ void cluster_probe_kernel() {}
}  // namespace

// Clusters of CL CTAs (one CTA per SM) that can be resident at once on the
// current device.  A cluster must fit in one GPC, so this is below num_sms/CL
// when GPC sizes are not multiples of CL; planning with num_sms/CL would then
// leave a second wave of clusters.  Cached per device.
int resident_clusters(int CL, int num_sms) {
  static std::mutex mu;
  static int cache[64][2] = {};
  int dev = 0;
  const int fallback = num_sms / CL;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || (CL != 4 && CL != 8)) {
    cudaGetLastError();
    return fallback;
  }
  const int slot = CL == 4 ? 0 : 1;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev][slot] == 0) {
    const int smem = 200 * 1024;  // forces one CTA per SM, like the recurrent kernels
    int n = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL * fallback);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaFuncSetAttribute(cluster_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, cluster_probe_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = fallback;
    }
    cache[dev][slot] = n < fallback ? n : fallback;
  }
  return cache[dev][slot];
}

RecPlan plan_recurrent(int B, int H, int num_sms, int force_wide, bool skip_zero) {
  RecPlan p{};
  p.HP = pad_neurons(H);
  if (skip_zero && !force_wide && p.HP <= 64) {
    plan_sparse(p, B, num_sms);
    return p;
  }
  if (skip_zero && !force_wide && H > 128) {
    p.HP = H <= 256 ? 256 : 512;
    plan_csparse(p, B, resident_clusters(8, num_sms));
    return p;
  }
  if (force_wide) {
    p.wide = true;
    plan_wide(p, B, H, num_sms);
    return p;
  }
  if (H > 128) {
    plan_stream(p, B, H, 8 * resident_clusters(8, num_sms));
    return p;
  }
  const int HP = p.HP;  // 32, 64 or 128
  const int LDV = HP + 4;
  const int CL = HP > 64 ? 4 : 1;  // cluster_of<HP>()
  const int groups = CL > 1 ? resident_clusters(CL, num_sms) : num_sms;
  const int blocks = (B + kSB - 1) / kSB;
  // each kernel: an equal share of sample blocks per resident sample group
  // shared-memory bound of the backward kernel (15 per-sample slabs + the reduction area)
  const size_t smem_cap = 227 * 1024 - 1024;
  const int max_per = (int)((smem_cap - 5 * HP * (HP / 8) * sizeof(float)) / (15 * LDV * sizeof(float) * kSB));
  // blocks per group: as many waves of resident groups as the per-group cap
  // forces, and the blocks spread evenly over them (a ragged last wave costs a
  // full one)
  const int cap = CL > 1 && max_per > kMaxBlk ? kMaxBlk : (max_per < 1 ? 1 : max_per);
  auto share = [&](int groups_per_pass) {
    const long long per_wave = (long long)groups_per_pass * cap;
    const long long waves = (blocks + per_wave - 1) / per_wave;
    const long long slots = waves * groups_per_pass;
    int per = (int)((blocks + slots - 1) / slots);
    if (per > cap) per = cap;
    if (per < 1) per = 1;
    return per * kSB;
  };
  const bool h64 = HP >= 64;
  p.ns_fwd = share(groups * (h64 ? LTC_FWD_CTAS : 1));
  p.ns_bwd = share(groups);
  p.grid_fwd = CL * ((B + p.ns_fwd - 1) / p.ns_fwd);
  p.grid_bwd = CL * ((B + p.ns_bwd - 1) / p.ns_bwd);
  p.threads_fwd = HP * HP / 8 / CL / (h64 ? LTC_FWD_RPT : 1);
  p.threads_bwd = HP * HP / 8 / CL / (HP >= 128 ? LTC_BWD_RPT128 : h64 ? LTC_BWD_RPT : 1);
  p.slots_bwd = p.grid_bwd / CL;
  p.smem_fwd = (size_t)6 * p.ns_fwd * LDV * sizeof(float);
  p.smem_bwd = ((size_t)15 * p.ns_bwd * LDV + 5 * HP * (HP / 8)) * sizeof(float);
  p.tanh_space = true;
  return p;
}

cudaError_t launch_recurrent_fwd(const RecFwdArgs& a, const RecPlan& p, cudaStream_t st) {
  if (p.sparse) return launch_sparse_fwd(a, p, a.tables, st);
  if (p.streamed) return launch_stream_fwd(a, p, st);
  if (p.wide) return launch_wide_fwd(a, p, st);
  switch (p.HP) {
    case 32: return launch_fast_fwd<32>(a, p, st);
    case 64: return launch_fast_fwd<64>(a, p, st);
    default: return launch_fast_fwd<128>(a, p, st);
  }
}

cudaError_t launch_recurrent_bwd(const RecBwdArgs& a, const RecPlan& p, cudaStream_t st) {
  if (p.sparse) return launch_sparse_bwd(a, p, a.tables, st);
  if (p.streamed) return launch_stream_bwd(a, p, st);
  if (p.wide) return launch_wide_bwd(a, p, st);
  switch (p.HP) {
    case 32: return launch_fast_bwd<32>(a, p, st);
    case 64: return launch_fast_bwd<64>(a, p, st);
    default: return launch_fast_bwd<128>(a, p, st);
  }
}

}  // namespace ltc

namespace ltc {
int read_wait_timeouts(int* count) {
  return (int)cudaMemcpyFromSymbol(count, g_ltc_wait_timeouts, sizeof(int));
}
}  // namespace ltc
