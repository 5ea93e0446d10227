// Cluster-streamed recurrent kernels for 128 < H <= 512 (padded to HP = 256 or 512).
//
// The dense H x H synapse set (4 gate-pack floats + 4 gradient sums per synapse:
// 8 MB at H = 512) fits in no CTA or cluster, so each 8-CTA cluster owns one
// group of `ns` samples and each CTA owns NEUR = HP/8 neurons:
//   forward : CTA = columns [nb, nb+NEUR); per unfold it streams the pack rows
//             (chunks of PC presynaptic rows x its columns) and the matching
//             slice of every sample's state through double-buffered shared
//             memory (cp.async), thread = (column, sample subgroup).
//   backward: CTA = rows [nb, nb+NEUR); per unfold it streams column chunks of
//             its pack rows and of its gradient slab (4 sums per synapse, kept in
//             L2: 4*NEUR*HP floats per CTA), thread = (row, 8 columns), and
//             accumulates every synapse over all ns samples in registers before
//             writing the chunk back -- one read-modify-write per synapse per
//             unfold for the whole sample group.  Its chunks (pack slice, 4 slab
//             tiles, a'_n / a'_d tiles) arrive by TMA tensor copies that one
//             thread issues, counted on an mbarrier per buffer, so the compute
//             warps never stall on copy issue; generic writes that a later TMA
//             reads are fenced with fence.proxy.async before the cluster barrier.
// Per-neuron vectors (state in the forward; a_n, a_d in the backward) are
// exchanged through global memory (L2) and ordered by the hardware cluster
// barrier (release/acquire at cluster scope), one barrier per unfold.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "ltc_cluster.cuh"
#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace cg = cooperative_groups;

namespace ltc {

// bounded waits of the streamed backward that expired (see ltc_cluster.cuh)
__device__ int g_stream_wait_timeouts = 0;


namespace {

constexpr int kCL = 8;    // CTAs per cluster
constexpr int kNT = 256;  // threads per CTA
constexpr int kPC = 32;   // presynaptic rows per forward chunk
constexpr int kSB = 4;    // samples per register block (backward)
constexpr int kMaxTailSamples = 96;

// Backward launch parameters: the scalar arguments plus the TMA descriptors of the
// four streamed operands (encoded on the host per launch; the kernel reads them
// from the grid-constant parameter space).
struct StreamBwdParams {
  RecBwdArgs a;
  CUtensorMap tm_pack;  // chunk-reordered gate pack (packT, see PackArgs::packT_qc) as
                        // [HP rows][4*HP floats]; box {4*QC, NEUR}
  CUtensorMap tm_slab;  // gradient slabs as [slots*4*HP rows][HP floats]; box {QC, NEUR}
  CUtensorMap tm_an;    // a'_n scratch as [2][B][HP] floats; box {QC, ns, 1} (rows >= B read 0)
  CUtensorMap tm_ad;    // a'_d scratch, same
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(tm), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)), "l"(tm), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
// generic-proxy global writes (slab write-back, adjoint scratch) before later
// async-proxy (TMA) reads of the same memory
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}  // samples per group the backward's tail handles (ns cap)

template <int NEUR>
struct SGeom {
  static constexpr int HP = NEUR * kCL;
  static constexpr int SGF = kNT / NEUR;  // forward sample subgroups
  static constexpr int QL = kNT / NEUR;   // backward lanes per row
  static constexpr int QC = QL * 8;       // backward columns per chunk
};

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// --------------------------------------------------------------------------- forward
template <int NEUR, int NSPT>
__global__ void __launch_bounds__(kNT, 1) rec_fwd_stream(RecFwdArgs a) {
  using G = SGeom<NEUR>;
  constexpr int HP = G::HP, SGF = G::SGF, NC = HP / kPC;
  extern __shared__ __align__(16) float smem[];
  const int ns = SGF * NSPT;
  float4* pks = reinterpret_cast<float4*>(smem);     // [2][kPC][NEUR]
  float* vch = smem + 2 * 4 * kPC * NEUR;            // [2][ns][kPC]

  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x;
  const int nb = (int)cluster.block_rank() * NEUR;
  const int ql = tid % NEUR, sg = tid / NEUR;
  const int q = nb + ql;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int b0 = (blockIdx.x / kCL) * ns;
  const int nvalid = min(ns, B - b0);
  float* vstate = a.scratch;  // [2][B][HP]
  const long long SB_ = (long long)B * HP;

  // per-column constants: 0.5 * sum_p w (the act = 0.5 + 0.5 tanh split)
  float ce = 0.f, cp = 0.f;
  for (int p = 0; p < HP; ++p) {
    const float4 w = a.pack[(long long)p * HP + q];
    ce += w.w;
    cp += w.z;
  }
  const float4 nq = a.nrn[q];
  const float cm = nq.x, cmgl = nq.x + nq.y, glvl = nq.w;
  const bool qvalid = q < H;

  // both state buffers: the padded neurons must read as 0 in every unfold
  for (int i = tid; i < nvalid * NEUR; i += kNT) {
    const int s = i / NEUR, h = nb + i % NEUR;
    const long long o = (long long)(b0 + s) * HP + h;
    vstate[o] = (a.h0 && h < H) ? a.h0[(long long)(b0 + s) * H + h] : 0.f;
    vstate[SB_ + o] = 0.f;
  }
  cluster.sync();

  auto stage = [&](int c, int buf, const float* vcur) {
    float4* dst = pks + buf * kPC * NEUR;
    for (int i = tid; i < kPC * NEUR; i += kNT) {
      const int pp = i / NEUR, cc = i % NEUR;
      cp_async16(dst + i, a.pack + (long long)(c * kPC + pp) * HP + nb + cc);
    }
    float* vd = vch + buf * ns * kPC;
    for (int i = tid; i < nvalid * (kPC / 4); i += kNT) {
      const int s = i / (kPC / 4), k4 = i % (kPC / 4);
      cp_async16(vd + s * kPC + 4 * k4, vcur + (long long)(b0 + s) * HP + c * kPC + 4 * k4);
    }
    cp_async_commit();
  };

  int cur = 0;
  for (int t = 0; t < T; ++t) {
    for (int u = 0; u < U; ++u) {
      const long long n = (long long)t * U + u;
      const float* vc = vstate + cur * SB_;
      float* vn = vstate + (cur ^ 1) * SB_;
      float2 an[NSPT], ad[NSPT];  // (even, odd) presynaptic rows, summed at the end
#pragma unroll
      for (int i = 0; i < NSPT; ++i) an[i] = ad[i] = make_float2(0.f, 0.f);
      stage(0, 0, vc);
      for (int c = 0; c < NC; ++c) {
        cp_async_wait_all();
        __syncthreads();
        if (c + 1 < NC) stage(c + 1, (c + 1) & 1, vc);
        const float4* pk = pks + (c & 1) * kPC * NEUR + ql;
        const float* vr = vch + (c & 1) * ns * kPC + sg * kPC;
#pragma unroll 2
        for (int pp = 0; pp < kPC; pp += 4) {
          const float4 w0 = pk[pp * NEUR], w1 = pk[(pp + 1) * NEUR];
          const float4 w2 = pk[(pp + 2) * NEUR], w3 = pk[(pp + 3) * NEUR];
          const float2 sx01 = make_float2(w0.x, w1.x), sy01 = make_float2(w0.y, w1.y);
          const float2 sz01 = make_float2(w0.z, w1.z), sw01 = make_float2(w0.w, w1.w);
          const float2 sx23 = make_float2(w2.x, w3.x), sy23 = make_float2(w2.y, w3.y);
          const float2 sz23 = make_float2(w2.z, w3.z), sw23 = make_float2(w2.w, w3.w);
#pragma unroll
          for (int i = 0; i < NSPT; ++i) {
            const float4 v4 = *reinterpret_cast<const float4*>(vr + i * SGF * kPC + pp);
            const float2 t01 = tanh2(fma2(sx01, make_float2(v4.x, v4.y), sy01));
            const float2 t23 = tanh2(fma2(sx23, make_float2(v4.z, v4.w), sy23));
            an[i] = fma2(sw23, t23, fma2(sw01, t01, an[i]));
            ad[i] = fma2(sz23, t23, fma2(sz01, t01, ad[i]));
          }
        }
      }
#pragma unroll
      for (int i = 0; i < NSPT; ++i) {
        const int s = sg + i * SGF;
        if (s < nvalid && qvalid) {
          const long long bs = b0 + s;
          const long long row = bs * T + t;
          const float v = vc[bs * HP + q];
          const float num = (cm * v + glvl) + (0.5f * (ce + (an[i].x + an[i].y)) + a.sn[row * H + q]);
          const float r = rcp_approx((cmgl + (0.5f * (cp + (ad[i].x + ad[i].y)) + a.sd[row * H + q])) + a.eps);
          const float vnew = num * r;
          vn[bs * HP + q] = vnew;
          if (a.V) {
            a.V[(n * B + bs) * H + q] = v;
            a.R[(n * B + bs) * H + q] = r;
          }
          if (u == U - 1 && a.out) a.out[row * H + q] = vnew;
        }
      }
      cluster.sync();  // release this unfold's states / acquire the peers'
      cur ^= 1;
    }
  }
  const float* vc = vstate + cur * SB_;
  for (int i = tid; i < nvalid * NEUR; i += kNT) {
    const int s = i / NEUR, h = nb + i % NEUR;
    if (h >= H) continue;
    const long long bs = b0 + s;
    if (a.hT) a.hT[bs * H + h] = vc[bs * HP + h];
    if (a.V) a.V[((long long)T * U * B + bs) * H + h] = vc[bs * HP + h];
  }
}

// --------------------------------------------------------------------------- backward
// scratch layout: AN, AD [2][B][HP] (by unfold parity), DIR, GSN, GSD [B][HP]
template <int NEUR>
__global__ void __launch_bounds__(kNT, 1) rec_bwd_stream(const __grid_constant__ StreamBwdParams P) {
  using G = SGeom<NEUR>;
  constexpr int HP = G::HP, QL = G::QL, QC = G::QC, NC = HP / QC;
  using LR = LaneReduce<QL, kSB>;
  const RecBwdArgs& a = P.a;
  extern __shared__ __align__(16) float smem_raw[];
  // TMA destinations must be 128-byte aligned
  float* smem = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int ns = a.ns;
  // chunk c of the CTA's rows, staged by TMA (one thread issues, an mbarrier per
  // buffer counts the bytes), dense row-major as in global memory
  float4* pks = reinterpret_cast<float4*>(smem);        // [2][NEUR][QC]  gate pack
  float* gch = smem + 2 * NEUR * QC * 4;                // [2][4][NEUR][QC] gradient sums
  float* anc = gch + 2 * 4 * NEUR * QC;                 // [2][ns][QC]  a'_n
  float* adc = anc + 2 * ns * QC;                       // [2][ns][QC]  a'_d
  float* DV = adc + 2 * ns * QC;                        // [ns][NEUR]
  float* VPb = DV + ns * NEUR;                          // [2][ns][NEUR]: V[m] of the own rows, slot m&1
  __shared__ __align__(8) uint64_t cbar[2];
  __shared__ int cabort;

  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31;
  const int nb = (int)cluster.block_rank() * NEUR;
  const int rl = tid / QL, ql = tid % QL;
  const int p = nb + rl;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int grp = blockIdx.x / kCL;
  const int b0 = grp * ns;
  const int nvalid = min(ns, B - b0);
  const int NTU = T * U;
  const long long SB_ = (long long)B * HP;
  float* ANg = a.scratch;
  float* ADg = ANg + 2 * SB_;
  float* DIRg = ADg + 2 * SB_;
  float* GSNg = DIRg + SB_;
  float* GSDg = GSNg + SB_;
  const long long hp2 = (long long)HP * HP;
  float* slab = a.part + (long long)grp * 4 * hp2;  // rows of the CTAs of a cluster are disjoint
  const float4 np_ = a.nrn[p];
  const float cm = np_.x, gl = np_.y, vl = np_.z;
  const bool pvalid = p < H;
  float gcm = 0.f, ggl = 0.f, gvl = 0.f, san = 0.f, sad = 0.f;

  // adjoint rows of padded samples (b >= B, last group only) arrive as zeros from
  // the TMA's out-of-range fill
  const int nblk = (nvalid + kSB - 1) / kSB;
  const uint32_t chunk_bytes = (uint32_t)(NEUR * QC * 16 + 4 * NEUR * QC * 4 + 2 * ns * QC * 4);
  if (tid == 0) {
    cabort = (smem_addr(smem) & 127u) != 0;  // never true with the rounding above
    mbar_init(smem_addr(&cbar[0]), 1);
    mbar_init(smem_addr(&cbar[1]), 1);
    mbar_init_fence();
  }
  // padded rows / samples of both V slots stay 0 (only valid entries are staged)
  for (int i = tid; i < 2 * ns * NEUR; i += kNT) VPb[i] = 0.f;
  __syncthreads();
  auto stage_vp = [&](int m) {  // V[m] -> VPb[m&1]
    float* dst = VPb + (m & 1) * ns * NEUR;
    const int nr = min(NEUR, H - nb);
    if (nr <= 0) return;
    for (int i = tid; i < nvalid * nr; i += kNT) {
      const int s = i / nr, r = i % nr;
      cp_async4(dst + s * NEUR + r, a.V + ((long long)m * B + b0 + s) * H + nb + r);
    }
  };
  stage_vp(NTU - 1);
  cp_async_commit();
  // zero this CTA's rows of the gradient slab (kept when accumulating segments)
  for (int i = tid; i < (a.accumulate ? 0 : NEUR * HP); i += kNT) {
    const long long o = (long long)(nb + i / HP) * HP + i % HP;
    slab[o] = 0.f;
    slab[hp2 + o] = 0.f;
    slab[2 * hp2 + o] = 0.f;
    slab[3 * hp2 + o] = 0.f;
  }

  // prep of unfold m for (sample s, own row p) given g = dL/dv_{m+1}[p]
  auto prep = [&](int m, int s, float gval, bool first) {
    const long long bs = b0 + s;
    const float r = a.R[((long long)m * B + bs) * H + p];
    const float vin = a.V[((long long)m * B + bs) * H + p];
    const float vout = a.V[((long long)(m + 1) * B + bs) * H + p];
    const float an = gval * r;
    const float ad = -an * vout;
    gcm = fmaf(an, vin - vout, gcm);
    ggl = fmaf(an, vl - vout, ggl);
    gvl = fmaf(an, gl, gvl);
    san += an;
    sad += ad;
    const long long o = bs * HP + p;
    GSNg[o] = first ? an : GSNg[o] + an;
    GSDg[o] = first ? ad : GSDg[o] + ad;
    DIRg[o] = an * cm;
    // the synapse pass works in tanh space: it reads a' = -a/4
    ANg[(m & 1) * SB_ + o] = -0.25f * an;
    ADg[(m & 1) * SB_ + o] = -0.25f * ad;
  };

  // initial prep of unfold NTU-1: g = dL/dout[:, T-1] + dL/dstate; padded rows write zeros
  for (int s = ql; s < ns; s += QL) {
    const long long bs = b0 + s;
    if (s >= nvalid) continue;
    if (pvalid) {
      float gval = a.gout[bs * a.go_sb + (long long)(T - 1) * a.go_st + (long long)p * a.go_sh];
      if (a.gstate) gval += a.gstate[bs * H + p];
      prep(NTU - 1, s, gval, true);
    } else {
      for (int par = 0; par < 2; ++par) {
        ANg[par * SB_ + bs * HP + p] = 0.f;
        ADg[par * SB_ + bs * HP + p] = 0.f;
      }
    }
  }
  cp_async_wait_all();  // V[NTU-1] of the own rows
  fence_proxy_async_global();  // slab zeros and adjoints before the TMA reads
  cluster.sync();

  auto stage = [&](int n, int c, int buf) {  // chunk c of unfold n -> buffer buf
    if (tid == 0 && !cabort) {
      const uint32_t bar = smem_addr(&cbar[buf]);
      mbar_arm(bar, chunk_bytes);
      tma_load_2d(pks + buf * NEUR * QC, &P.tm_pack, c * QC * 4, nb, bar);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        tma_load_2d(gch + (buf * 4 + k) * NEUR * QC, &P.tm_slab, c * QC, (grp * 4 + k) * HP + nb, bar);
      tma_load_3d(anc + buf * ns * QC, &P.tm_an, c * QC, b0, n & 1, bar);
      tma_load_3d(adc + buf * ns * QC, &P.tm_ad, c * QC, b0, n & 1, bar);
    }
  };
  uint32_t cphase = 0;  // parity bit per buffer

  const int own = LR::own_base(lane);
  const bool writer = LR::writer(lane);
  const float2 m1 = make_float2(-1.f, -1.f);
  int t = T - 1, k = U - 1;
  for (int n = NTU - 1; n >= 0; --n) {
    for (int i = tid; i < ns * NEUR; i += kNT) DV[i] = 0.f;
    const float* VP = VPb + (n & 1) * ns * NEUR;       // V[n], staged one unfold ahead
    const float* VPm = VPb + ((n + 1) & 1) * ns * NEUR;  // V[n-1], staged now for the tails
    if (n >= 1) {
      stage_vp(n - 1);
      cp_async_commit();
    }
    stage(n, 0, 0);
    for (int c = 0; c < NC; ++c) {
      const int buf = c & 1;
      mbar_wait(smem_addr(&cbar[buf]), (cphase >> buf) & 1u, &cabort, &g_stream_wait_timeouts);
      cphase ^= 1u << buf;
      __syncthreads();  // everyone is past chunk c-1: its buffer takes chunk c+1
      if (c + 1 < NC) stage(n, c + 1, (c + 1) & 1);
      float2 sl2[4], nm2[4], wp2[4], we2[4], G0[4], G1[4], G2[4], G3[4];
      // reordered chunk: synapse j of lane ql at j*QL + ql (2-way bank conflicts at most)
      const float4* pk = pks + buf * NEUR * QC + rl * QC + ql;
      const float* gs = gch + buf * 4 * NEUR * QC + rl * QC + ql * 8;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 p0 = pk[(2 * kk) * QL], p1 = pk[(2 * kk + 1) * QL];
        // negated half-scale constants: the gate argument is -z/2, so tanh gives -t
        sl2[kk] = make_float2(-p0.x, -p1.x);
        nm2[kk] = make_float2(-p0.y, -p1.y);
        wp2[kk] = make_float2(p0.z, p1.z);
        we2[kk] = make_float2(p0.w, p1.w);
      }
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const float4 g0 = *reinterpret_cast<const float4*>(gs + 4 * h2);
        const float4 g1 = *reinterpret_cast<const float4*>(gs + NEUR * QC + 4 * h2);
        const float4 g2 = *reinterpret_cast<const float4*>(gs + 2 * NEUR * QC + 4 * h2);
        const float4 g3 = *reinterpret_cast<const float4*>(gs + 3 * NEUR * QC + 4 * h2);
        G0[2 * h2] = make_float2(g0.x, g0.y); G0[2 * h2 + 1] = make_float2(g0.z, g0.w);
        G1[2 * h2] = make_float2(g1.x, g1.y); G1[2 * h2 + 1] = make_float2(g1.z, g1.w);
        G2[2 * h2] = make_float2(g2.x, g2.y); G2[2 * h2 + 1] = make_float2(g2.z, g2.w);
        G3[2 * h2] = make_float2(g3.x, g3.y); G3[2 * h2 + 1] = make_float2(g3.z, g3.w);
      }
      const float* ans = anc + buf * ns * QC + ql * 8;
      const float* ads = adc + buf * ns * QC + ql * 8;
      const float* vps = VP + rl;
      float* dvs = DV + own * NEUR + rl;
      for (int blk = 0; blk < nblk; ++blk, ans += kSB * QC, ads += kSB * QC, vps += kSB * NEUR,
               dvs += kSB * NEUR) {
        float acc[1][kSB];
#pragma unroll
        for (int i = 0; i < kSB; ++i) {
          const float4 a0 = *reinterpret_cast<const float4*>(ans + i * QC);
          const float4 a1 = *reinterpret_cast<const float4*>(ans + i * QC + 4);
          const float4 d0 = *reinterpret_cast<const float4*>(ads + i * QC);
          const float4 d1 = *reinterpret_cast<const float4*>(ads + i * QC + 4);
          const float2 an2[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                                 make_float2(a1.z, a1.w)};
          const float2 ad2[4] = {make_float2(d0.x, d0.y), make_float2(d0.z, d0.w), make_float2(d1.x, d1.y),
                                 make_float2(d1.z, d1.w)};
          const float vp = vps[i * NEUR];
          const float2 vp2 = make_float2(vp, vp);
          float2 dv = make_float2(0.f, 0.f);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // tanh space (as in the register-resident backward): tn = tanh(-z/2),
            // staged a' = -a/4:  dL/dz = (a'_n w_erev + a'_d w_pos)(tn^2 - 1),
            // a act = a/2 + 2 a' tn (the a/2 part comes from the per-row sums)
            const float2 tn = tanh2(fma2(sl2[kk], vp2, nm2[kk]));
            const float2 dz = mul2(fma2(an2[kk], we2[kk], mul2(ad2[kk], wp2[kk])), fma2(tn, tn, m1));
            G0[kk] = fma2(an2[kk], tn, G0[kk]);
            G1[kk] = fma2(ad2[kk], tn, G1[kk]);
            G2[kk] = add2(G2[kk], dz);
            G3[kk] = fma2(dz, vp2, G3[kk]);
            dv = fma2(dz, sl2[kk], dv);
          }
          acc[0][i] = dv.x + dv.y;
        }
        LR::template run<1>(acc, lane);
        if (writer && blk * kSB + own < nvalid) *dvs += acc[0][0];
      }
      // write the chunk's gradient sums back to the slab (L2)
      float* gdst = slab + (long long)p * HP + c * QC + ql * 8;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int k0 = 2 * h2, k1 = 2 * h2 + 1;
        *reinterpret_cast<float4*>(gdst + 4 * h2) = make_float4(G0[k0].x, G0[k0].y, G0[k1].x, G0[k1].y);
        *reinterpret_cast<float4*>(gdst + hp2 + 4 * h2) = make_float4(G1[k0].x, G1[k0].y, G1[k1].x, G1[k1].y);
        *reinterpret_cast<float4*>(gdst + 2 * hp2 + 4 * h2) = make_float4(G2[k0].x, G2[k0].y, G2[k1].x, G2[k1].y);
        *reinterpret_cast<float4*>(gdst + 3 * hp2 + 4 * h2) = make_float4(G3[k0].x, G3[k0].y, G3[k1].x, G3[k1].y);
      }
    }
    cp_async_wait_all();  // V[n-1] for the tails
    __syncthreads();
    // per-neuron tails of the own rows, samples s = ql + j*QL.  All global loads
    // of the thread's samples are issued first (the chunk registers are dead
    // here), then the math and stores run: the L2 latencies overlap instead of
    // serialising behind the stores of the previous sample.
    {
      constexpr int kTS = kMaxTailSamples / QL;
      const bool last = (k == 0 && t == 0);  // unfold 0 of step 0: only dL/dh0 remains
      float dirv[kTS], gsnv[kTS], gsdv[kTS], rv[kTS], gov[kTS];
#pragma unroll
      for (int j = 0; j < kTS; ++j) {
        const int s = ql + j * QL;
        dirv[j] = gsnv[j] = gsdv[j] = rv[j] = gov[j] = 0.f;
        if (s < nvalid && pvalid) {
          const long long bs = b0 + s;
          const long long o = bs * HP + p;
          dirv[j] = ldcg(DIRg + o);
          gsnv[j] = ldcg(GSNg + o);
          gsdv[j] = ldcg(GSDg + o);
          if (!last) rv[j] = a.R[((long long)(n - 1) * B + bs) * H + p];
          if (k == 0 && !last) gov[j] = a.gout[bs * a.go_sb + (long long)(t - 1) * a.go_st + (long long)p * a.go_sh];
        }
      }
#pragma unroll
      for (int j = 0; j < kTS; ++j) {
        const int s = ql + j * QL;
        if (s < nvalid && pvalid) {
          const long long bs = b0 + s;
          const long long o = bs * HP + p;
          float gval = fmaf(-2.0f, DV[s * NEUR + rl], dirv[j]);  // sl holds -sigma/2
          if (k == 0) {
            const long long row = bs * T + t;
            a.gsn[row * H + p] = gsnv[j];
            a.gsd[row * H + p] = gsdv[j];
            if (last) {
              a.gh0[bs * H + p] = gval;
              continue;
            }
            gval += gov[j];
          }
          // prep of unfold n-1: R[n-1], V[n-1] (VPm) and V[n] (VP)
          const float r = rv[j];
          const float vin = VPm[s * NEUR + rl];
          const float vout = VP[s * NEUR + rl];
          const float an = gval * r;
          const float ad = -an * vout;
          gcm = fmaf(an, vin - vout, gcm);
          ggl = fmaf(an, vl - vout, ggl);
          gvl = fmaf(an, gl, gvl);
          san += an;
          sad += ad;
          const bool first = k == 0;
          GSNg[o] = first ? an : gsnv[j] + an;
          GSDg[o] = first ? ad : gsdv[j] + ad;
          DIRg[o] = an * cm;
          ANg[((n - 1) & 1) * SB_ + o] = -0.25f * an;
          ADg[((n - 1) & 1) * SB_ + o] = -0.25f * ad;
        }
      }
    }
    fence_proxy_async_global();  // slab write-back and a'_n/a'_d before the TMA reads
    cluster.sync();  // release a_n/a_d of unfold n-1 / acquire the peers'
    if (--k < 0) {
      k = U - 1;
      --t;
    }
  }
  // per-neuron partial sums: reduce over the QL lanes of the row (fixed order)
#pragma unroll
  for (int stride = QL / 2; stride >= 1; stride >>= 1) {
    gcm += __shfl_xor_sync(0xffffffffu, gcm, stride);
    ggl += __shfl_xor_sync(0xffffffffu, ggl, stride);
    gvl += __shfl_xor_sync(0xffffffffu, gvl, stride);
    san += __shfl_xor_sync(0xffffffffu, san, stride);
    sad += __shfl_xor_sync(0xffffffffu, sad, stride);
  }
  if (ql == 0) {  // 5 rows: the tanh-space layout (+ sum a_n, sum a_d per neuron)
    float* pn = a.partn + (long long)grp * 5 * HP;
    const float v[5] = {gcm, ggl, gvl, san, sad};
#pragma unroll
    for (int k = 0; k < 5; ++k) pn[k * HP + p] = a.accumulate ? pn[k * HP + p] + v[k] : v[k];
  }
}

template <typename Args>
cudaError_t launch_cluster8(void (*kernel)(Args), const Args& a, int grid, size_t smem, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int NEUR>
cudaError_t fwd_dispatch(const RecFwdArgs& a, const RecPlan& p, cudaStream_t st) {
#define LTC_NSPT_CASE(N) \
  case N: return launch_cluster8(rec_fwd_stream<NEUR, N>, a, p.grid_fwd, p.smem_fwd, st);
  switch (p.ns_fwd / SGeom<NEUR>::SGF) {
    LTC_NSPT_CASE(1) LTC_NSPT_CASE(2) LTC_NSPT_CASE(3) LTC_NSPT_CASE(4) LTC_NSPT_CASE(6)
    LTC_NSPT_CASE(8) LTC_NSPT_CASE(12) LTC_NSPT_CASE(16) LTC_NSPT_CASE(18) LTC_NSPT_CASE(20)
    LTC_NSPT_CASE(24)
    default: return cudaErrorInvalidConfiguration;
  }
#undef LTC_NSPT_CASE
}

}  // namespace

void plan_stream(RecPlan& p, int B, int H, int num_sms) {
  const int HP = H <= 256 ? 256 : 512;
  const int NEUR = HP / kCL;
  const int SGF = kNT / NEUR, QC = (kNT / NEUR) * 8;
  p.HP = HP;
  p.wide = true;
  p.streamed = true;
  const int groups = num_sms / kCL > 0 ? num_sms / kCL : 1;  // resident clusters
  // samples per group: at most what the backward's shared memory holds (its
  // staging grows by 16*QC + 12*NEUR bytes per sample), in steps of SGF samples
  // per thread of the forward (instantiated counts kNspt); as many waves of
  // resident clusters as that cap forces, the samples spread evenly over them
  constexpr int kNspt[] = {1, 2, 3, 4, 6, 8, 12, 16, 18, 20, 24};
  constexpr int kNn = sizeof(kNspt) / sizeof(kNspt[0]);
  const long long fixed = (long long)2 * NEUR * QC * 16 + (long long)2 * 4 * NEUR * QC * 4 + 128;
  int ns_cap = (int)((227LL * 1024 - 1024 - fixed) / (16 * QC + 12 * NEUR));
  if (ns_cap > kMaxTailSamples) ns_cap = kMaxTailSamples;
  int top = 0;  // largest instantiated count within the cap
  for (int i = 0; i < kNn; ++i)
    if (kNspt[i] * SGF <= ns_cap) top = i;
  const long long per_wave = (long long)groups * kNspt[top] * SGF;
  const long long waves = (B + per_wave - 1) / per_wave;
  const int want = (int)((B + waves * groups - 1) / (waves * groups));
  int nspt = kNspt[top];
  for (int i = top; i >= 0; --i)
    if (kNspt[i] * SGF >= want) nspt = kNspt[i];
  const int ns = nspt * SGF;  // a multiple of kSB
  p.ns_fwd = p.ns_bwd = ns;
  const int ngroups = (B + ns - 1) / ns;
  p.grid_fwd = p.grid_bwd = ngroups * kCL;
  p.threads_fwd = p.threads_bwd = kNT;
  p.slots_bwd = ngroups;
  p.smem_fwd = (size_t)2 * kPC * NEUR * 16 + (size_t)2 * ns * kPC * 4;
  p.smem_bwd = (size_t)fixed + (size_t)4 * ns * QC * 4 +
               (size_t)3 * ns * NEUR * 4;
  p.tanh_space = true;
  p.scratch_fwd = (size_t)2 * B * HP;
  p.scratch_bwd = (size_t)7 * B * HP;
}

cudaError_t launch_stream_fwd(const RecFwdArgs& a, const RecPlan& p, cudaStream_t st) {
  return p.HP == 256 ? fwd_dispatch<32>(a, p, st) : fwd_dispatch<64>(a, p, st);
}

namespace {
// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    cudaGetLastError();
  });
  return fn;
}

bool encode_f32(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                const cuuint32_t* box) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u)) return false;
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_stream_bwd(const RecBwdArgs& a, const RecPlan& p, cudaStream_t st) {
  const int HP = p.HP, NEUR = HP / kCL, QC = (kNT / NEUR) * 8;
  const int slots = p.grid_bwd / kCL;
  StreamBwdParams P;
  memset(&P, 0, sizeof(P));
  P.a = a;
  const float* ANg = a.scratch;
  const float* ADg = ANg + 2 * (size_t)a.B * HP;
  const cuuint64_t dp[2] = {(cuuint64_t)HP * 4, (cuuint64_t)HP};
  const cuuint64_t sp[1] = {(cuuint64_t)HP * 16};
  const cuuint32_t bp[2] = {(cuuint32_t)QC * 4, (cuuint32_t)NEUR};
  const cuuint64_t ds[2] = {(cuuint64_t)HP, (cuuint64_t)slots * 4 * HP};
  const cuuint64_t ss[1] = {(cuuint64_t)HP * 4};
  const cuuint32_t bs[2] = {(cuuint32_t)QC, (cuuint32_t)NEUR};
  const cuuint64_t da[3] = {(cuuint64_t)HP, (cuuint64_t)a.B, 2};
  const cuuint64_t sa[2] = {(cuuint64_t)HP * 4, (cuuint64_t)a.B * HP * 4};
  const cuuint32_t ba[3] = {(cuuint32_t)QC, (cuuint32_t)a.ns, 1};
  if (!a.packT || !encode_f32(&P.tm_pack, a.packT, 2, dp, sp, bp) || !encode_f32(&P.tm_slab, a.part, 2, ds, ss, bs) ||
      !encode_f32(&P.tm_an, ANg, 3, da, sa, ba) || !encode_f32(&P.tm_ad, ADg, 3, da, sa, ba))
    return cudaErrorInvalidValue;  // no launch with a descriptor that did not encode
  return HP == 256 ? launch_cluster8(rec_bwd_stream<32>, P, p.grid_bwd, p.smem_bwd, st)
                   : launch_cluster8(rec_bwd_stream<64>, P, p.grid_bwd, p.smem_bwd, st);
}

int read_stream_wait_timeouts(int* count) {
  return (int)cudaMemcpyFromSymbol(count, g_stream_wait_timeouts, sizeof(int));
}


}  // namespace ltc
