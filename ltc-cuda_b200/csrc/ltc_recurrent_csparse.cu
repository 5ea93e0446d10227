// Zero-synapse-skipping recurrent kernels for 128 < H <= 512 (LTC_FLAG_SKIP_ZERO_SYNAPSES).
//
// Same contract as the H <= 64 skipping kernels (ltc_recurrent_sparse.cu): only
// synapses whose w_pos or w_erev is nonzero are visited; the four recurrent
// gradients are left unwritten (the finish kernel writes zeros) at the others.
//
// Geometry.  An 8-CTA cluster owns a group of ns samples; CTA r owns NEUR = HP/8
// neurons (columns in the forward, rows in the backward) and keeps their nonzero
// synapse lists resident in shared memory for the whole sequence -- at density 0.2
// and H = 512 about 6.5 K synapses per CTA, 100 KB of gate constants -- so nothing
// is re-streamed per unfold except the per-neuron vectors, which go through L2
// (global scratch, neuron-major) and are ordered by one cluster barrier per unfold.
//
// Forward: a warp takes one column; lane = (sample quad, list part): each lane runs
// 4 samples of a staged 32-sample slice per list entry (one float4 gather of the
// presynaptic states, the entry's constants a shared-memory broadcast), the list is
// split over 32 / quads parts, and a transposed shuffle reduction over the parts
// leaves one (column, sample) sum per owner lane.
// Backward: 8 lanes share a pair of rows (the c-th heaviest and the c-th lightest
// by count); a lane holds up to 32 slots of the pair's synapses with their 4
// gradient sums in registers for the whole sequence and their constants in shared
// memory; samples come in chunks of 8, the adjoints of all HP columns for the chunk
// staged neuron-major (odd float4 stride) and gathered per synapse; the
// per-(row, sample) sum dL/dv is reduced over the 8 lanes by the transposed
// reduction.  A warp's slot counts (K1, K2) run as compile-time constants.
// The saved V / R of this path are neuron-major (see below).
//
// Capacity: at most 8192 nonzero synapses enter each CTA's block of HP/8 columns;
// inside each block of HP/8 rows, with the rows ranked by count and paired c-th
// heaviest with c-th lightest in warps of 4 pairs, a warp needs K1 + K2 <= 32 slots
// (K1 = 4*ceil(max ceil(heavy/8) / 4), K2 likewise for the light rows).  The table
// builder flags a violation and the kernels then write NaN to their outputs
// (ltc_cuda.skip_zero_synapses_fits applies the same rule on the host).
#include <cooperative_groups.h>

#include <cstdint>
#include <type_traits>

#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace cg = cooperative_groups;

namespace ltc {
namespace {

constexpr int kCL = 8;        // CTAs per cluster
constexpr int kNT = 256;      // threads per CTA (backward)
constexpr int kNTF = 512;     // threads per CTA (forward: 16 warps hide the list walk's latencies)
constexpr int kFCap = 8192;   // forward: synapses per CTA (its column block)
constexpr int kBK = 32;       // backward: synapses per lane (both rows of its pair)
constexpr int kBL = 8;        // backward lanes per row pair
constexpr int kSB = 4;        // backward samples per register block
constexpr int kCS = 8;        // backward samples per staged chunk (= kBL: one tail sample per lane)
constexpr int kCS4 = 3;       // float4 per neuron in a staged adjoint chunk (odd, >= kCS/4)
constexpr int kFS = 32;       // forward samples per staged slice (one per lane)

// tables in the caller's workspace, per cluster rank r (see csp_tables_bytes)
struct CspTables {
  int* fcoff;       // [8][NEUR + 1]   forward: list offsets of the CTA's columns
  uint16_t* fent;   // [8][kFCap]      presynaptic neuron of each entry
  int* brow;        // [8][NEUR]       backward: row of lane group g (rows ranked by count)
  int* bk;          // [8][8]          slots per lane of each warp (multiple of 4)
  uint16_t* bidx;   // [8][kBK][kNT]   postsynaptic neuron of (slot, thread); 0xFFFF = padding
  int* overflow;    // [1]
};

inline size_t csp_layout(int HP, size_t (&at)[6]) {
  const int NEUR = HP / kCL;
  const size_t sz[6] = {(size_t)kCL * (NEUR + 1) * sizeof(int), (size_t)kCL * kFCap * sizeof(uint16_t),
                        (size_t)kCL * NEUR * sizeof(int), (size_t)kCL * 8 * sizeof(int),
                        (size_t)kCL * kBK * kNT * sizeof(uint16_t), sizeof(int)};
  size_t o = 0;
  for (int i = 0; i < 6; ++i) {
    at[i] = o;
    o = (o + sz[i] + 255) & ~size_t(255);
  }
  return o;
}

inline CspTables csp_view(void* base, int HP) {
  char* b = static_cast<char*>(base);
  size_t at[6];
  csp_layout(HP, at);
  CspTables t;
  t.fcoff = reinterpret_cast<int*>(b + at[0]);
  t.fent = reinterpret_cast<uint16_t*>(b + at[1]);
  t.brow = reinterpret_cast<int*>(b + at[2]);
  t.bk = reinterpret_cast<int*>(b + at[3]);
  t.bidx = reinterpret_cast<uint16_t*>(b + at[4]);
  t.overflow = reinterpret_cast<int*>(b + at[5]);
  return t;
}

__device__ inline bool nonzero(const float* wp, const float* we, long long j) { return wp[j] != 0.f || we[j] != 0.f; }

// ---- table builder: grid (8 ranks, 2 sides), 256 threads ----------------------
template <int HP>
__global__ void __launch_bounds__(kNT) build_csp_kernel(CspTables tb, const float* __restrict__ w_pos,
                                                        const float* __restrict__ w_erev, int H) {
  constexpr int NEUR = HP / kCL, NW = HP / 32;
  const int r = blockIdx.x, side = blockIdx.y, tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nb = r * NEUR;
  __shared__ uint32_t nzm[NEUR][NW];  // nonzero partners of each own neuron, as bits
  __shared__ int cnt[NEUR];
  __shared__ int order[NEUR];
  // bits: backward (side 0) row p = nb + i over columns q; forward (side 1) column
  // q = nb + i over rows p; one warp per neuron, a ballot per 32 partners
  for (int i = warp; i < NEUR; i += kNT / 32) {
    const int n = nb + i;
    int c = 0;
    for (int h = 0; h < NW; ++h) {
      const int o = 32 * h + lane;
      const long long j = side ? (long long)o * H + n : (long long)n * H + o;
      const bool on = n < H && o < H && nonzero(w_pos, w_erev, j);
      const uint32_t m = __ballot_sync(0xffffffffu, on);
      if (lane == 0) nzm[i][h] = m;
      c += __popc(m);
    }
    if (lane == 0) cnt[i] = c;
  }
  __syncthreads();
  if (side == 1) {  // forward: CSR over the CTA's columns, partners ascending
    if (tid == 0) {
      int o = 0;
      for (int i = 0; i < NEUR; ++i) {
        tb.fcoff[r * (NEUR + 1) + i] = min(o, kFCap);
        o += cnt[i];
      }
      tb.fcoff[r * (NEUR + 1) + NEUR] = min(o, kFCap);
      if (o > kFCap) atomicOr(tb.overflow, 1);
    }
    __syncthreads();
    for (int i = warp; i < NEUR; i += kNT / 32) {
      int base = tb.fcoff[r * (NEUR + 1) + i];
      for (int h = 0; h < NW; ++h) {
        const uint32_t m = nzm[i][h];
        const bool on = (m >> lane) & 1u;
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        if (on && pos < kFCap) tb.fent[r * kFCap + pos] = (uint16_t)(32 * h + lane);
        base += __popc(m);
      }
    }
    return;
  }
  // backward: rows ranked by count; lane group c (8 lanes) takes the c-th heaviest
  // (A) and the c-th lightest (B) row; a warp (4 groups) runs K1 slots of its A rows
  // and K2 of its B rows (multiples of 4, K1 + K2 <= kBK)
  for (int i = tid; i < NEUR; i += kNT) {
    int rk = 0;
    for (int m = 0; m < NEUR; ++m) rk += (cnt[m] > cnt[i]) || (cnt[m] == cnt[i] && m < i);
    order[rk] = i;
  }
  __syncthreads();
  constexpr int NPAIR = NEUR / 2, NWB = NPAIR / 4;  // pairs; warps holding pairs
  // pair group g (4 rank-consecutive pairs) -> warp: with 8 warps, groups 2s and 2s+1
  // (similar slot counts) share scheduler s (warps s and s + 4), so each scheduler runs
  // at most a couple of the compile-time variants and their code stays in its cache
  auto warp_of = [](int g) { return NWB == 8 ? ((g & 1) ? 4 + g / 2 : g / 2) : g; };
  __shared__ int k1w[8], k2w[8];
  for (int g = tid; g < 8; g += kNT) {
    const int w = g < NWB ? warp_of(g) : g;
    int k1 = 0, k2 = 0;
    for (int c = 4 * g; c < 4 * g + 4 && g < NWB; ++c) {
      k1 = max(k1, (cnt[order[c]] + kBL - 1) / kBL);
      k2 = max(k2, (cnt[order[NEUR - 1 - c]] + kBL - 1) / kBL);
    }
    k1 = (k1 + 3) & ~3;
    k2 = (k2 + 3) & ~3;
    if (k1 + k2 > kBK) {
      atomicOr(tb.overflow, 1);
      k2 = max(0, kBK - k1);
      k1 = min(k1, kBK);
    }
    k1w[w] = k1;
    k2w[w] = k2;
    tb.bk[r * 8 + w] = k1 | (k2 << 8);
  }
  for (int i = tid; i < NEUR; i += kNT) {  // rows of pair slot ps = warp * 4 + c % 4
    const int c = i / 2, ps = warp_of(c / 4) * 4 + c % 4;
    tb.brow[r * NEUR + 2 * ps + (i & 1)] = nb + order[(i & 1) ? NEUR - 1 - c : c];
  }
  __syncthreads();
  // entries: a row's partners round-robin over the residues mod 8 (bank spread of
  // the gathers); entry e of row A -> lane e % 8, slot e / 8; of row B -> slot K1 + e / 8
  for (int i = tid; i < kBK * NPAIR * kBL; i += kNT)  // padding first
    tb.bidx[(size_t)r * kBK * kNT + (i / (NPAIR * kBL)) * kNT + i % (NPAIR * kBL)] = 0xFFFFu;
  __syncthreads();
  for (int k = tid; k < NEUR; k += kNT) {
    const int c = k / 2, rsel = k % 2, w = warp_of(c / 4), ps = w * 4 + c % 4;
    const int row = order[rsel ? NEUR - 1 - c : c];
    const int base = rsel ? k1w[w] : 0, lim = rsel ? k2w[w] : k1w[w];
    if (cnt[row] > kBL * lim) atomicOr(tb.overflow, 1);
    uint64_t cls[8];
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) cls[bb] = 0;
    for (int h = 0; h < NW; ++h) {
      uint32_t m = nzm[row][h];
      while (m) {
        const int q = 32 * h + __ffs(m) - 1;
        m &= m - 1;
#pragma unroll
        for (int bb = 0; bb < 8; ++bb)
          if ((q & 7) == bb) cls[bb] |= 1ull << (q >> 3);
      }
    }
    int e = 0;
    bool more = true;
    while (more && e < kBL * lim) {
      more = false;
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) {
        if (cls[bb] && e < kBL * lim) {
          const int j = __ffsll((long long)cls[bb]) - 1;
          cls[bb] &= cls[bb] - 1;
          tb.bidx[(size_t)r * kBK * kNT + (base + e / kBL) * kNT + ps * kBL + e % kBL] = (uint16_t)(8 * j + bb);
          ++e;
          more = true;
        }
      }
    }
  }
}

// Saved state.  On this path V and R are stored neuron-major per unfold,
// V[n][q][b] (n in [0, T*U], the last slice the final state) and R[n][q][b]: the
// forward's owner lanes are consecutive samples of one neuron, so its stores and the
// backward's staging reads are contiguous.  Only these two kernels read or write it.

// ---- forward --------------------------------------------------------------------
// scratch: vstate [2][HP][BP] neuron-major (BP = planned sample capacity)
template <int NEUR>
__global__ void __launch_bounds__(kNTF, 1) rec_fwd_csp(RecFwdArgs a, CspTables tb, int BP) {
  constexpr int HP = NEUR * kCL;
  extern __shared__ __align__(16) float smem[];
  float4* cst = reinterpret_cast<float4*>(smem);                          // [kFCap]
  float* vs = smem + 4 * kFCap;                                             // [HP][kFS]
  uint16_t* ent = reinterpret_cast<uint16_t*>(vs + HP * kFS);               // [kFCap]
  int* coff = reinterpret_cast<int*>(ent + kFCap);                          // [NEUR + 1]
  float* cw = reinterpret_cast<float*>(coff + NEUR + 1);                    // [2][NEUR]

  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int r = (int)cluster.block_rank(), nb = r * NEUR;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int ns = a.ns, b0 = (blockIdx.x / kCL) * ns;
  const int nvalid = min(ns, B - b0);
  const int nsg = (nvalid + kFS - 1) / kFS;
  float* vstate = a.scratch;
  const long long SV = (long long)HP * BP;
  const bool bad = *tb.overflow != 0;

  for (int i = tid; i <= NEUR; i += kNTF) coff[i] = tb.fcoff[r * (NEUR + 1) + i];
  __syncthreads();
  // constants of the own columns' synapses (sigma/2, -sigma*mu/2, w_pos/2, w_erev/2)
  for (int c = warp; c < NEUR; c += kNTF / 32) {
    const int q = nb + c;
    float se = 0.f, sp = 0.f;
    for (int e = coff[c] + lane; e < coff[c + 1]; e += 32) {
      if (LTC_CHECKED_SKIP(e >= 0 && e < kFCap, 201)) continue;
      int p = tb.fent[r * kFCap + e];
      if (LTC_CHECKED_SKIP(p >= 0 && p < HP, 202)) p = 0;
      float4 k = a.pack[(long long)p * HP + q];
      k.z *= 0.5f;
      k.w *= 0.5f;
      cst[e] = k;
      ent[e] = (uint16_t)p;
      se += k.w;
      sp += k.z;
    }
    for (int o = 16; o >= 1; o >>= 1) {
      se += __shfl_xor_sync(0xffffffffu, se, o);
      sp += __shfl_xor_sync(0xffffffffu, sp, o);
    }
    if (lane == 0) {
      cw[c] = se;
      cw[NEUR + c] = sp;
    }
  }
  // initial states of the own columns
  for (int i = tid; i < NEUR * nvalid; i += kNTF) {
    const int c = i / nvalid, s = i % nvalid, q = nb + c;
    vstate[(long long)q * BP + b0 + s] = (a.h0 && q < H) ? a.h0[(long long)(b0 + s) * H + q] : 0.f;
  }
  __syncthreads();
  cluster.sync();

  int cur = 0;
  for (int t = 0; t < T; ++t) {
    for (int u = 0; u < U; ++u) {
      const long long n = (long long)t * U + u;
      const float* vc = vstate + cur * SV;
      float* vn = vstate + (cur ^ 1) * SV;
      for (int g = 0; g < nsg; ++g) {
        const int sb = b0 + g * kFS;  // first sample of the slice (reads past B are never used)
        const int cnt = min(kFS, nvalid - g * kFS);
        const int n4 = (cnt + 3) / 4;  // float4 per neuron that hold the slice's samples
        for (int i = tid; i < HP * n4; i += kNTF) {
          const int p = i / n4, k4 = i % n4;
          cp_async16(vs + p * kFS + 4 * k4, vc + (long long)p * BP + sb + 4 * k4);
        }
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
        // Lane = (sample quad sq, list part): each lane runs 4 samples per synapse
        // entry (one float4 gather, the entry's constants loaded once), the column's
        // list is split over F = 32 / SQ parts (SQ = quads in the slice, a power of
        // two, so a short slice still fills the warp), and a transposed shuffle
        // reduction over the parts leaves one sample of the column per owner lane.
        const int SQ = cnt <= 4 ? 1 : cnt <= 8 ? 2 : cnt <= 16 ? 4 : 8, F = 32 / SQ;
        const int sq = lane % SQ, part = lane / SQ;
        const bool hA = part & (F / 2), hB = part & (F / 4);
        const bool lead = (part & (F / 4 - 1)) == 0;
        const int s = g * kFS + 4 * sq + 2 * hA + hB;  // the sample this lane owns if lead
        for (int c = warp; c < NEUR; c += kNTF / 32) {
          const int q = nb + c;
          // the tail's global reads are issued before the synapse pass hides their latency
          const bool owner = lead && s < nvalid && q < H;
          const long long row = (long long)(b0 + s) * T + t;
          float snv = 0.f, sdv = 0.f;
          float4 nq = make_float4(0.f, 0.f, 0.f, 0.f);
          if (owner) {
            snv = a.sn[row * H + q];
            sdv = a.sd[row * H + q];
            nq = a.nrn[q];
          }
          float an[4] = {0.f, 0.f, 0.f, 0.f}, ad[4] = {0.f, 0.f, 0.f, 0.f};
          auto visit = [&](int e) {
            const float4 k = cst[e];
            const float4 v = *reinterpret_cast<const float4*>(vs + ent[e] * kFS + 4 * sq);
            const float th[4] = {tanh_approx(fmaf(k.x, v.x, k.y)), tanh_approx(fmaf(k.x, v.y, k.y)),
                                 tanh_approx(fmaf(k.x, v.z, k.y)), tanh_approx(fmaf(k.x, v.w, k.y))};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              an[i] = fmaf(k.w, th[i], an[i]);
              ad[i] = fmaf(k.z, th[i], ad[i]);
            }
          };
          int e = coff[c] + part;
          const int e1 = coff[c + 1];
          for (; e + F < e1; e += 2 * F) {
            visit(e);
            visit(e + F);
          }
          if (e < e1) visit(e);
          // parts F/2 apart: keep samples (2, 3) or (0, 1), send the other pair
          float a2[2], d2[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float sa = hA ? an[i] : an[2 + i], sd_ = hA ? ad[i] : ad[2 + i];
            a2[i] = (hA ? an[2 + i] : an[i]) + __shfl_xor_sync(0xffffffffu, sa, 16);
            d2[i] = (hA ? ad[2 + i] : ad[i]) + __shfl_xor_sync(0xffffffffu, sd_, 16);
          }
          // parts F/4 apart: keep one sample of the pair
          float an1 = (hB ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, hB ? a2[0] : a2[1], 8);
          float ad1 = (hB ? d2[1] : d2[0]) + __shfl_xor_sync(0xffffffffu, hB ? d2[0] : d2[1], 8);
          for (int off = SQ; off < 8; off *= 2) {  // the remaining part bits: plain sums
            an1 += __shfl_xor_sync(0xffffffffu, an1, off);
            ad1 += __shfl_xor_sync(0xffffffffu, ad1, off);
          }
          if (owner && !LTC_CHECKED_SKIP(b0 + s < B && b0 + s < BP && q < HP, 203)) {
            const long long bs = b0 + s;
            const float v = vs[q * kFS + (s - g * kFS)];
            const float num = (nq.x * v + nq.w) + ((cw[c] + an1) + snv);
            const float rr = rcp_approx((nq.x + nq.y) + ((cw[NEUR + c] + ad1) + sdv) + a.eps);
            const float vnew = bad ? __int_as_float(0x7fc00000) : num * rr;
            vn[(long long)q * BP + bs] = vnew;
            if (a.V) {
              a.V[(n * H + q) * B + bs] = v;  // neuron-major saved state (this path's own layout)
              a.R[(n * H + q) * B + bs] = rr;
            }
            if (u == U - 1 && a.out) a.out[row * H + q] = vnew;
          }
        }
        __syncthreads();  // the slice buffer is restaged next
      }
      cluster.sync();  // release this unfold's states / acquire the peers'
      cur ^= 1;
    }
  }
  const float* vc = vstate + cur * SV;
  for (int i = tid; i < NEUR * nvalid; i += kNTF) {
    const int c = i / nvalid, s = i % nvalid, q = nb + c;
    if (q >= H) continue;
    const long long bs = b0 + s;
    const float v = vc[(long long)q * BP + bs];
    if (a.hT) a.hT[bs * H + q] = v;
    if (a.V) a.V[((long long)T * U * H + q) * B + bs] = v;
  }
  cluster.sync();  // no CTA leaves while a peer may still read its states
}

// ---- backward -------------------------------------------------------------------
// scratch: AN, AD [2][HP][BP] neuron-major (by unfold parity); DIR, GSN, GSD [HP][B]
struct CspBwd {
  float Gwe[kBK], Gwp[kBK], Gdz[kBK], Gdzv[kBK];

  // slots [J0, J0 + K) of the lane, all of one row with states vr (4 samples):
  // dv[i] += dL/dz * (-sigma/2)
  template <int J0, int K>
  __device__ __forceinline__ void run(const float4* __restrict__ cst, const uint16_t* __restrict__ qix,
                                      const float* an_b, const float* ad_b, const float4& vr, float (&dv)[kSB],
                                      int tid) {
    const float v[4] = {vr.x, vr.y, vr.z, vr.w};
#pragma unroll
    for (int j = J0; j < J0 + K; ++j) {
      const float4 k = cst[j * kNT + tid];  // (-sigma/2, sigma*mu/2, w_pos, w_erev)
      const int q = qix[j * kNT + tid];
      const float4 a4 = *reinterpret_cast<const float4*>(an_b + q * (4 * kCS4));
      const float4 d4 = *reinterpret_cast<const float4*>(ad_b + q * (4 * kCS4));
      const float an[4] = {a4.x, a4.y, a4.z, a4.w}, ad[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
      for (int i = 0; i < kSB; ++i) {
        // tanh space, as in the dense kernels: tn = tanh(-z/2), a' = -a/4
        const float tn = tanh_approx(fmaf(k.x, v[i], k.y));
        const float dz = fmaf(an[i], k.w, ad[i] * k.z) * fmaf(tn, tn, -1.f);
        Gwe[j] = fmaf(an[i], tn, Gwe[j]);
        Gwp[j] = fmaf(ad[i], tn, Gwp[j]);
        Gdz[j] += dz;
        Gdzv[j] = fmaf(dz, v[i], Gdzv[j]);
        dv[i] = fmaf(dz, k.x, dv[i]);
      }
    }
  }

  // one block of 4 samples: acc[0][r * 4 + i] for row r (A, B) and sample i
  template <int K1, int K2>
  __device__ __forceinline__ void pass(const float4* cst, const uint16_t* qix, const float* an_b,
                                       const float* ad_b, const float4 (&vr)[2], float (&acc)[1][2 * kSB],
                                       int tid) {
    float dv[2][kSB];
#pragma unroll
    for (int i = 0; i < kSB; ++i) dv[0][i] = dv[1][i] = 0.f;
    run<0, K1>(cst, qix, an_b, ad_b, vr[0], dv[0], tid);
    run<K1, K2>(cst, qix, an_b, ad_b, vr[1], dv[1], tid);
#pragma unroll
    for (int i = 0; i < kSB; ++i) {
      acc[0][i] = dv[0][i];
      acc[0][kSB + i] = dv[1][i];
    }
  }
};

// warp's (K1, K2), multiples of 4 with K1 >= K2 and K1 + K2 <= kBK -> compile-time pass
template <typename Fn>
__device__ __forceinline__ void csp_dispatch(int kw, Fn&& fn) {
  switch (kw) {
#define LTC_CSP(K1, K2) \
  case (K1) | ((K2) << 8): fn(std::integral_constant<int, K1>{}, std::integral_constant<int, K2>{}); return;
    LTC_CSP(0, 0) LTC_CSP(4, 0) LTC_CSP(4, 4) LTC_CSP(8, 0) LTC_CSP(8, 4) LTC_CSP(8, 8) LTC_CSP(12, 0)
    LTC_CSP(12, 4) LTC_CSP(12, 8) LTC_CSP(12, 12) LTC_CSP(16, 0) LTC_CSP(16, 4) LTC_CSP(16, 8) LTC_CSP(16, 12)
    LTC_CSP(16, 16) LTC_CSP(20, 0) LTC_CSP(20, 4) LTC_CSP(20, 8) LTC_CSP(20, 12) LTC_CSP(24, 0) LTC_CSP(24, 4)
    LTC_CSP(24, 8) LTC_CSP(28, 0) LTC_CSP(28, 4)
#undef LTC_CSP
    default: fn(std::integral_constant<int, kBK>{}, std::integral_constant<int, 0>{}); return;
  }
}

template <int NEUR>
__global__ void __launch_bounds__(kNT, 1) rec_bwd_csp(RecBwdArgs a, CspTables tb, int BP) {
  constexpr int HP = NEUR * kCL, NPAIR = NEUR / 2;
  using LR = LaneReduce<kBL, 2 * kSB>;
  extern __shared__ __align__(16) float smem[];
  float4* cst = reinterpret_cast<float4*>(smem);                     // [kBK][kNT]
  float* anc = smem + 4 * kBK * kNT;                                   // [HP][4 * kCS4]
  float* adc = anc + HP * 4 * kCS4;                                    // [HP][4 * kCS4]
  // per chunk, double-buffered: V[n], V[n-1], R[n-1], DIR, GSN, GSD of the own rows
  float* tdat = adc + HP * 4 * kCS4;                                   // [2][6][NEUR][kCS]
  uint16_t* qix = reinterpret_cast<uint16_t*>(tdat + 2 * 6 * NEUR * kCS);  // [kBK][kNT]
  float* dvb = reinterpret_cast<float*>(qix + kBK * kNT);              // [NEUR][kCS]  dL/dv of the chunk
  int* rowof = reinterpret_cast<int*>(dvb + NEUR * kCS);               // [NEUR]  row of slot 2c + r

  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid / 32;
  const int r = (int)cluster.block_rank(), nb = r * NEUR;
  const int c = tid / kBL, l = tid % kBL;  // row pair and lane in the pair
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int grp = blockIdx.x / kCL;
  const int ns = a.ns, b0 = grp * ns;
  const int nvalid = min(ns, B - b0);
  const int nch = (nvalid + kCS - 1) / kCS;
  const int NTU = T * U;
  const long long SV = (long long)HP * BP;
  float* ANg = a.scratch;
  float* ADg = ANg + 2 * SV;
  float* DIRg = ADg + 2 * SV;
  float* GSNg = DIRg + (long long)B * HP;
  float* GSDg = GSNg + (long long)B * HP;
  const float bad = *tb.overflow ? __int_as_float(0x7fc00000) : 0.f;
  const bool active = c < NPAIR;  // NEUR = 32: threads 128..255 hold no rows
  const int kw = active ? tb.bk[r * 8 + warp] : 0;
  const int K1w = kw & 0xFF;
  const int rowA = active ? tb.brow[r * NEUR + 2 * c] : nb;
  const int rowB = active ? tb.brow[r * NEUR + 2 * c + 1] : nb;
  auto prow = [&](int rsel) { return rsel ? rowB : rowA; };
  if (tid < NEUR) rowof[tid] = tb.brow[r * NEUR + tid];

  // the lane's synapse constants (-sigma/2, sigma*mu/2, w_pos, w_erev) and columns;
  // padding slots get zero constants and read column 0
  for (int j = 0; j < kBK; ++j) {
    uint16_t q = active ? tb.bidx[(size_t)r * kBK * kNT + j * kNT + tid] : (uint16_t)0xFFFF;
    if (q != 0xFFFF && LTC_CHECKED_SKIP(q < HP, 211)) q = 0xFFFF;
    float4 k = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q != 0xFFFF) {
      k = a.pack[(long long)prow(j < K1w ? 0 : 1) * HP + q];
      k.x = -k.x;
      k.y = -k.y;
    }
    cst[j * kNT + tid] = k;
    qix[j * kNT + tid] = q == 0xFFFF ? 0 : q;
  }
  CspBwd f;
#pragma unroll
  for (int j = 0; j < kBK; ++j) f.Gwe[j] = f.Gwp[j] = f.Gdz[j] = f.Gdzv[j] = bad;
  float4 nrn2[2];
  nrn2[0] = a.nrn[prow(0)];
  nrn2[1] = a.nrn[prow(1)];
  float sums[2][5];  // per row: g_cm, g_gl, g_vl, sum a_n, sum a_d
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int kk = 0; kk < 5; ++kk) sums[rr][kk] = bad;
  const int own = LR::own_base(lane);  // item (row own / 4, sample own % 4) of a block

  // prep of unfold m for (sample bs, row rsel) given g = dL/dv_{m+1}
  auto prep = [&](int rsel, int m, long long bs, float gval, bool first, float vin, float vout, float rr,
                  float gsn_prev, float gsd_prev) {
    const int p = prow(rsel);
    const float an = gval * rr;
    const float ad = -an * vout;
    sums[rsel][0] = fmaf(an, vin - vout, sums[rsel][0]);
    sums[rsel][1] = fmaf(an, nrn2[rsel].z - vout, sums[rsel][1]);
    sums[rsel][2] = fmaf(an, nrn2[rsel].y, sums[rsel][2]);
    sums[rsel][3] += an;
    sums[rsel][4] += ad;
    const long long o = (long long)p * B + bs;  // neuron-major, like the saved state
    GSNg[o] = first ? an : gsn_prev + an;
    GSDg[o] = first ? ad : gsd_prev + ad;
    DIRg[o] = an * nrn2[rsel].x;
    ANg[(m & 1) * SV + (long long)p * BP + bs] = -0.25f * an;
    ADg[(m & 1) * SV + (long long)p * BP + bs] = -0.25f * ad;
  };

  // initial prep of unfold NTU-1 (g = dL/dout[:, T-1] + dL/dstate); padded rows write zeros
  if (active) {
#pragma unroll
    for (int rsel = 0; rsel < 2; ++rsel) {
      const int p = prow(rsel);
      for (int s = l; s < nvalid; s += kBL) {
        const long long bs = b0 + s;
        if (p < H) {
          float gval = a.gout[bs * a.go_sb + (long long)(T - 1) * a.go_st + (long long)p * a.go_sh];
          if (a.gstate) gval += a.gstate[bs * H + p];
          const long long m = NTU - 1;
          prep(rsel, NTU - 1, bs, gval, true, a.V[(m * H + p) * B + bs], a.V[((m + 1) * H + p) * B + bs],
               a.R[(m * H + p) * B + bs], 0.f, 0.f);
        } else {
          for (int par = 0; par < 2; ++par) {
            ANg[par * SV + (long long)p * BP + bs] = 0.f;
            ADg[par * SV + (long long)p * BP + bs] = 0.f;
          }
        }
      }
    }
  }
  __syncthreads();
  cluster.sync();

  int t = T - 1, k = U - 1;
  for (int n = NTU - 1; n >= 0; --n) {
    const float* ANn = ANg + (n & 1) * SV;
    const float* ADn = ADg + (n & 1) * SV;
    const bool last = (k == 0 && t == 0);
    // staging of chunk ch into the adjoint buffers (free while no pass runs) and
    // tail buffer tb_: everything the chunk's pass and tails read, so the tails
    // wait on no global load
    auto stage = [&](int ch, int tbuf) {
      const int sc = ch * kCS;
      for (int i = tid; i < HP * (kCS / 4); i += kNT) {
        const int q = i / (kCS / 4), k4 = i % (kCS / 4);
        cp_async16(anc + q * 4 * kCS4 + 4 * k4, ANn + (long long)q * BP + b0 + sc + 4 * k4);
        cp_async16(adc + q * 4 * kCS4 + 4 * k4, ADn + (long long)q * BP + b0 + sc + 4 * k4);
      }
      float* td = tdat + tbuf * 6 * NEUR * kCS;
      // every field of a full chunk is kCS contiguous samples per row (neuron-major
      // saved state and scratch): 16-byte copies when every row stays aligned
      const bool vec = (B & 3) == 0 && sc + kCS <= nvalid &&
                       ((reinterpret_cast<uintptr_t>(a.V) | reinterpret_cast<uintptr_t>(a.R) |
                         reinterpret_cast<uintptr_t>(DIRg)) & 15) == 0;
      const int f0 = vec ? 6 : 0;  // first field of the per-element loop
      if (vec) {
        for (int i = tid; i < 6 * NEUR * (kCS / 4); i += kNT) {
          const int fld = i / (NEUR * (kCS / 4)), rs = (i / (kCS / 4)) % NEUR, k4 = i % (kCS / 4);
          const int row = rowof[rs];
          float* dst = td + (fld * NEUR + rs) * kCS + 4 * k4;
          if (row < H && (fld == 0 || fld >= 3 || !last)) {
            const long long bs = b0 + sc + 4 * k4;
            const float* src = fld == 0 ? a.V + ((long long)n * H + row) * B + bs
                             : fld == 1 ? a.V + ((long long)(n - 1) * H + row) * B + bs
                             : fld == 2 ? a.R + ((long long)(n - 1) * H + row) * B + bs
                             : fld == 3 ? DIRg + (long long)row * B + bs
                             : fld == 4 ? GSNg + (long long)row * B + bs
                                        : GSDg + (long long)row * B + bs;
            cp_async16(dst, src);
          } else {
            *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      for (int i = tid + f0 * NEUR * kCS; i < 6 * NEUR * kCS; i += kNT) {
        const int fld = i / (NEUR * kCS), rs = (i / kCS) % NEUR, sl = i % kCS;
        const int row = rowof[rs];
        const long long bs = b0 + sc + sl;
        const bool ok = sc + sl < nvalid && row < H && (fld == 0 || fld >= 3 || !last);
        const float* src;
        switch (fld) {
          case 0: src = a.V + ((long long)n * H + row) * B + bs; break;
          case 1: src = a.V + ((long long)(n - 1) * H + row) * B + bs; break;
          case 2: src = a.R + ((long long)(n - 1) * H + row) * B + bs; break;
          case 3: src = DIRg + (long long)row * B + bs; break;
          case 4: src = GSNg + (long long)row * B + bs; break;
          default: src = GSDg + (long long)row * B + bs; break;
        }
        cp_async4_zfill(td + i, ok ? src : a.V, ok);
      }
      cp_async_commit();
    };
    stage(0, 0);
    for (int ch = 0; ch < nch; ++ch) {
      const int sc = ch * kCS;  // first sample of the chunk (in the group)
      const float* td = tdat + (ch & 1) * 6 * NEUR * kCS;
      cp_async_wait_all();
      __syncthreads();
      if (sc + kCS > nvalid) {  // samples past the group's last: their adjoints must not count
        const int v0 = nvalid - sc;
        for (int i = tid; i < HP * (kCS - v0); i += kNT) {
          const int q = i / (kCS - v0), s = v0 + i % (kCS - v0);
          anc[q * 4 * kCS4 + s] = 0.f;
          adc[q * 4 * kCS4 + s] = 0.f;
        }
        __syncthreads();
      }
      for (int blk = 0; blk < kCS / kSB; ++blk) {
        float acc[1][2 * kSB];
        float4 vr[2];
#pragma unroll
        for (int rsel = 0; rsel < 2; ++rsel)
          vr[rsel] = active ? *reinterpret_cast<const float4*>(td + (2 * c + rsel) * kCS + blk * kSB)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        const float* an_b = anc + blk * kSB;
        const float* ad_b = adc + blk * kSB;
        csp_dispatch(kw, [&](auto K1, auto K2) {
          f.template pass<decltype(K1)::value, decltype(K2)::value>(cst, qix, an_b, ad_b, vr, acc, tid);
        });
        LR::template run<1>(acc, lane);
        if (active && !LTC_CHECKED_SKIP(2 * c + own / kSB < NEUR, 212))
          dvb[(2 * c + own / kSB) * kCS + blk * kSB + own % kSB] = acc[0][0];
      }
      __syncthreads();  // adjoint buffers free: the next chunk streams in behind the tails
      if (ch + 1 < nch) stage(ch + 1, (ch + 1) & 1);
      // tails of the chunk: lane l takes sample sc + l of both rows
      if (active) {
        const int s = sc + l;
        const long long bs = b0 + s;
        float gov[2] = {0.f, 0.f};
#pragma unroll
        for (int rsel = 0; rsel < 2; ++rsel) {
          const int p = prow(rsel);
          if (s < nvalid && p < H && !last && k == 0)
            gov[rsel] = a.gout[bs * a.go_sb + (long long)(t - 1) * a.go_st + (long long)p * a.go_sh];
        }
#pragma unroll
        for (int rsel = 0; rsel < 2; ++rsel) {
          const int p = prow(rsel);
          if (s >= nvalid || p >= H) continue;
          const int ti = (2 * c + rsel) * kCS + l;
          const float dirv = td[3 * NEUR * kCS + ti], gsnv = td[4 * NEUR * kCS + ti], gsdv = td[5 * NEUR * kCS + ti];
          float gval = fmaf(-2.0f, dvb[ti], dirv);  // the constants hold -sigma/2
          if (k == 0) {
            const long long row = bs * T + t;
            a.gsn[row * H + p] = gsnv;
            a.gsd[row * H + p] = gsdv;
            if (last) {
              a.gh0[bs * H + p] = gval;
              continue;
            }
            gval += gov[rsel];
          }
          prep(rsel, n - 1, bs, gval, k == 0, td[NEUR * kCS + ti], td[ti], td[2 * NEUR * kCS + ti], gsnv, gsdv);
        }
      }
    }
    cluster.sync();  // release a'_n / a'_d of unfold n-1 / acquire the peers'
    if (--k < 0) {
      k = U - 1;
      --t;
    }
  }
  // synapse partials at their dense positions (skipped synapses are never written)
  if (active) {
    float* part = a.part + (long long)grp * 4 * HP * HP;
    const long long hp2 = (long long)HP * HP;
#pragma unroll
    for (int j = 0; j < kBK; ++j) {
      const uint16_t q = tb.bidx[(size_t)r * kBK * kNT + j * kNT + tid];
      if (q == 0xFFFF || LTC_CHECKED_SKIP(q < HP, 213)) continue;
      const long long idx = (long long)prow(j < K1w ? 0 : 1) * HP + q;
      if (a.accumulate) {
        part[idx] += f.Gwe[j];
        part[hp2 + idx] += f.Gwp[j];
        part[2 * hp2 + idx] += f.Gdz[j];
        part[3 * hp2 + idx] += f.Gdzv[j];
      } else {
        part[idx] = f.Gwe[j];
        part[hp2 + idx] = f.Gwp[j];
        part[2 * hp2 + idx] = f.Gdz[j];
        part[3 * hp2 + idx] = f.Gdzv[j];
      }
    }
  }
  // per-neuron sums over the pair's lanes (fixed order)
#pragma unroll
  for (int stride = kBL / 2; stride >= 1; stride >>= 1)
#pragma unroll
    for (int rsel = 0; rsel < 2; ++rsel)
#pragma unroll
      for (int kk = 0; kk < 5; ++kk) sums[rsel][kk] += __shfl_xor_sync(0xffffffffu, sums[rsel][kk], stride);
  if (active && l < 2) {
    const int p = prow(l);
    float* pn = a.partn + (long long)grp * 5 * HP;
#pragma unroll
    for (int kk = 0; kk < 5; ++kk) {
      const float v = l ? sums[1][kk] : sums[0][kk];
      pn[kk * HP + p] = a.accumulate ? pn[kk * HP + p] + v : v;
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still read its adjoints
}

template <typename Kern, typename Args>
cudaError_t launch_c8(Kern kernel, const Args& a, const CspTables& tb, int BP, int grid, int threads, size_t smem,
                      cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a, tb, BP);
}

// sample capacity of the neuron-major scratch: every group's slices / chunks may
// read up to kFS samples past its own start
inline int csp_bp(const RecPlan& p) { return (p.grid_fwd / kCL) * p.ns_fwd + kFS; }

}  // namespace

size_t csp_tables_bytes(int HP) {
  size_t at[6];
  return csp_layout(HP, at);
}

void plan_csparse(RecPlan& p, int B, int num_clusters) {
  const int HP = p.HP;  // 256 or 512
  const int NEUR = HP / kCL;
  const int groups = num_clusters > 0 ? num_clusters : 1;
  int ns = (B + groups - 1) / groups;
  ns = (ns + kSB - 1) / kSB * kSB;
  p.sparse = true;
  p.streamed = true;
  p.wide = true;
  p.ns_fwd = p.ns_bwd = ns;
  p.grid_fwd = p.grid_bwd = ((B + ns - 1) / ns) * kCL;
  p.threads_fwd = kNTF;
  p.threads_bwd = kNT;
  p.slots_bwd = p.grid_bwd / kCL;
  p.smem_fwd = (size_t)kFCap * 16 + (size_t)HP * kFS * 4 + (size_t)kFCap * 2 + (NEUR + 1) * 4 + 2 * NEUR * 4;
  p.smem_bwd = (size_t)kBK * kNT * 16 + (size_t)2 * HP * 4 * kCS4 * 4 + (size_t)2 * 6 * NEUR * kCS * 4 +
               (size_t)kBK * kNT * 2 + (size_t)NEUR * kCS * 4 + NEUR * 4;
  p.tanh_space = true;
  const size_t BP = (size_t)(p.grid_fwd / kCL) * ns + kFS;
  p.scratch_fwd = 2 * (size_t)HP * BP;
  p.scratch_bwd = 4 * (size_t)HP * BP + 3 * (size_t)B * HP;
}

cudaError_t launch_build_csp(const PackArgs& pa, void* tables, cudaStream_t st) {
  const CspTables tb = csp_view(tables, pa.HP);
  cudaError_t e = cudaMemsetAsync(tb.overflow, 0, sizeof(int), st);
  if (e != cudaSuccess) return e;
  if (pa.HP == 512)
    build_csp_kernel<512><<<dim3(kCL, 2), kNT, 0, st>>>(tb, pa.w_pos, pa.w_erev, pa.H);
  else
    build_csp_kernel<256><<<dim3(kCL, 2), kNT, 0, st>>>(tb, pa.w_pos, pa.w_erev, pa.H);
  return cudaGetLastError();
}

cudaError_t launch_csp_fwd(const RecFwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st) {
  const CspTables tb = csp_view(const_cast<void*>(tables), p.HP);
  return p.HP == 512 ? launch_c8(rec_fwd_csp<64>, a, tb, csp_bp(p), p.grid_fwd, kNTF, p.smem_fwd, st)
                     : launch_c8(rec_fwd_csp<32>, a, tb, csp_bp(p), p.grid_fwd, kNTF, p.smem_fwd, st);
}

cudaError_t launch_csp_bwd(const RecBwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st) {
  const CspTables tb = csp_view(const_cast<void*>(tables), p.HP);
  return p.HP == 512 ? launch_c8(rec_bwd_csp<64>, a, tb, csp_bp(p), p.grid_bwd, kNT, p.smem_bwd, st)
                     : launch_c8(rec_bwd_csp<32>, a, tb, csp_bp(p), p.grid_bwd, kNT, p.smem_bwd, st);
}

}  // namespace ltc
