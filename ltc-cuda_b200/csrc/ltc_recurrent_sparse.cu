// Recurrent kernels that skip structurally-zero synapses (H <= 64, LTC_FLAG_SKIP_ZERO_SYNAPSES).
//
// A synapse whose w_pos and w_erev are both zero adds nothing to the solve
// (num/den terms are w * act) and has dL/dz = 0, so it only contributes to the
// gradients of w_pos / w_erev at its own position -- which a module that builds
// w_pos = softplus(w) * mask multiplies by zero.  With the flag the caller
// declares those gradients unused; these kernels then visit only the nonzero
// synapses and the finish kernel writes zeros at the skipped positions.
//
// Layout.  TPC = 8 lanes share a PAIR of
// neurons (rows in the backward, columns in the forward): the c-th heaviest and
// the c-th lightest by nonzero count, so every pair carries a similar total.
// Each lane holds up to KM synapses of each neuron, taken from the neuron's
// nonzero list (entry e -> lane e % TPC, slot e / TPC); a warp runs its slot
// counts (K1, K2) -- the largest of its heavy / light neurons' ceil(count / TPC)
// -- as compile-time constants, chosen by a jump table at the top of each sample
// block, so no per-slot branch is issued.
// The per-neuron vectors the synapse pass gathers from (v in the forward, the
// adjoints in the backward) are stored neuron-major, four samples per float4,
// with an odd number of float4 per neuron; lists are ordered round-robin over the
// residue mod 8, so the eight lanes of a quarter-warp (consecutive entries of one
// neuron's list) gather from distinct bank groups.  The packed f32x2 pairs run over two SAMPLES of one
// synapse (adjacent in the gathered float4), with the synapse constants
// duplicated in both halves, so forming the pairs costs no register moves.
//
// Capacity: at most 48 nonzero synapses per neuron at HP = 64 (TPC * KM); any
// mask at HP = 32.  The table builder checks it; a
// call whose mask exceeds it writes NaN to every output of the kernels (state,
// outputs, gradients) instead of a wrong number -- callers check the mask first
// (ltc_cuda.skip_zero_synapses does).
//
// Tables are rebuilt on the device at every call (build_slots_kernel, one CTA, a few
// microseconds),
// so the host never reads the mask and CUDA-graph capture stays possible.
#include <cstdint>
#include <type_traits>

#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace ltc {
namespace {

constexpr int kSB = 4;   // samples per block (one float4 of a neuron-major vector)
// lanes per neuron pair and slots per neuron and lane, forward (side 1) and backward
// (side 0): 8 lanes per pair (256 threads at HP = 64; one reduced item per lane in
// the tails; 16 lanes per pair in the forward measured the same at c3 and 3% slower
// at 4 samples per CTA).  Capacity is 48 synapses per neuron at HP = 64 and 32 (every
// mask) at HP = 32.
constexpr int kCap64 = 48;
__host__ __device__ constexpr int side_tpc(int) { return 8; }
__host__ __device__ constexpr int side_km(int HP, int side) { return (HP == 64 ? kCap64 : 32) / side_tpc(side); }
__host__ __device__ constexpr int side_nt(int HP, int side) { return HP / 2 * side_tpc(side); }

// slot tables inside the caller's workspace (see sparse_tables_bytes): neuron
// assignments and synapse lists only; the kernels read each slot's constants from
// the dense gate pack (pack[p][q]) once at start, so the tables depend on the
// nonzero pattern alone
struct SlotTablesView {
  int* fneu;      // [HP]          neuron of (pair c, r) at 2c + r (forward: column q)
  int* fk;        // [warps]       K1 | K2 << 8
  int* fidx;      // [NTf][2][KMf] presynaptic neuron p, -1 = padding
  int* bneu;      // [HP]          backward: row p
  int* bk;        // [warps]
  int* bidx;      // [NTb][2][KMb] postsynaptic neuron q, -1 = padding
  int* overflow;  // [1]           1 if a neuron has more nonzero synapses than the capacity
};

__host__ __device__ inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

// byte offsets of the table arrays; returns the total size
inline size_t tables_layout(int HP, size_t (&at)[7]) {
  const size_t nf = (size_t)side_nt(HP, 1) * 2 * side_km(HP, 1), nb = (size_t)side_nt(HP, 0) * 2 * side_km(HP, 0);
  const size_t sz[7] = {HP * sizeof(int), side_nt(HP, 1) / 32 * sizeof(int), nf * sizeof(int), HP * sizeof(int),
                        side_nt(HP, 0) / 32 * sizeof(int), nb * sizeof(int), sizeof(int)};
  size_t o = 0;
  for (int i = 0; i < 7; ++i) {
    at[i] = o;
    o = align_up(o + sz[i]);
  }
  return o;
}

inline SlotTablesView tables_view(void* base, int HP) {
  char* b = static_cast<char*>(base);
  size_t at[7];
  tables_layout(HP, at);
  SlotTablesView v;
  v.fneu = reinterpret_cast<int*>(b + at[0]);
  v.fk = reinterpret_cast<int*>(b + at[1]);
  v.fidx = reinterpret_cast<int*>(b + at[2]);
  v.bneu = reinterpret_cast<int*>(b + at[3]);
  v.bk = reinterpret_cast<int*>(b + at[4]);
  v.bidx = reinterpret_cast<int*>(b + at[5]);
  v.overflow = reinterpret_cast<int*>(b + at[6]);
  return v;
}

// ---- table builder: one CTA of 256 threads ---------------------------------
// Backward: neuron = row p, list = its nonzero columns q.  Forward: neuron =
// column q, list = its nonzero rows p.
template <int HP>
__global__ void __launch_bounds__(256) build_slots_kernel(SlotTablesView tv, const float* __restrict__ w_pos,
                                                          const float* __restrict__ w_erev, int ld, int rows,
                                                          int cols, int nqc, size_t chunk_bytes) {
  // One CTA per HP x HP block of a row-major (rows, cols) pattern with row stride ld,
  // blocks numbered (row block, column block) with nqc column blocks; block b's tables
  // sit chunk_bytes * b into the table area.  The recurrent matrix is one block
  // (rows = cols = ld = H); the sensory one (D, H) is cut into blocks for its backward.
  constexpr int NPAIR = HP / 2, CAP = HP == 64 ? kCap64 : 32;
  const int p0 = (blockIdx.x / nqc) * HP, q0 = (blockIdx.x % nqc) * HP;
  const int P = min(HP, rows - p0), Q = min(HP, cols - q0);
  w_pos += (long long)p0 * ld + q0;
  w_erev += (long long)p0 * ld + q0;
  if (blockIdx.x) {
    const size_t o = (size_t)blockIdx.x * chunk_bytes;
    auto sh = [o](int* ptr) { return reinterpret_cast<int*>(reinterpret_cast<char*>(ptr) + o); };
    tv.fneu = sh(tv.fneu);
    tv.fk = sh(tv.fk);
    tv.fidx = sh(tv.fidx);
    tv.bneu = sh(tv.bneu);
    tv.bk = sh(tv.bk);
    tv.bidx = sh(tv.bidx);
    tv.overflow = sh(tv.overflow);
  }
  __shared__ uint64_t nz[2][HP];  // [0] bit q of row p; [1] bit p of column q
  __shared__ int cnt[2][HP];
  __shared__ int order[2][HP];    // neurons by count, descending
  __shared__ unsigned char lst[2][HP][HP];  // each neuron's list (neuron indices), in emission order
  const int tid = threadIdx.x;
  // nonzero pattern: one warp per row, a ballot per 32 columns (coalesced loads, no atomics)
  const int warp = tid / 32, lane = tid % 32, nwarps = blockDim.x / 32;
  for (int p = warp; p < HP; p += nwarps) {
    uint64_t m = 0;
#pragma unroll
    for (int h = 0; h < HP / 32; ++h) {
      const int q = 32 * h + lane;
      const long long j = (long long)p * ld + q;
      const bool on = p < P && q < Q && (w_pos[j] != 0.f || w_erev[j] != 0.f);
      m |= (uint64_t)__ballot_sync(0xffffffffu, on) << (32 * h);
    }
    if (lane == 0) nz[0][p] = m;
  }
  __syncthreads();
  for (int p = tid; p < HP; p += blockDim.x) cnt[0][p] = __popcll(nz[0][p]);
  for (int q = tid; q < HP; q += blockDim.x) {
    uint64_t m = 0;
    for (int p = 0; p < HP; ++p)
      if ((nz[0][p] >> q) & 1ull) m |= 1ull << p;
    nz[1][q] = m;
    cnt[1][q] = __popcll(m);
  }
  __syncthreads();
  for (int i = tid; i < 2 * HP; i += blockDim.x) {  // stable rank by count, descending
    const int s = i / HP, n = i % HP, c = cnt[s][n];
    int r = 0;
    for (int m = 0; m < HP; ++m) r += (cnt[s][m] > c) || (cnt[s][m] == c && m < n);
    order[s][r] = n;
  }
  __syncthreads();
  if (tid == 0) {
    int over = 0;
    for (int i = 0; i < 2 * HP; ++i) over |= cnt[i / HP][i % HP] > CAP;
    *tv.overflow = over;
  }
  // neuron of (pair c, r): r = 0 the c-th heaviest, r = 1 the c-th lightest
  for (int i = tid; i < 2 * HP; i += blockDim.x) {
    const int s = i / HP, k = i % HP, c = k / 2, r = k % 2;
    (s ? tv.fneu : tv.bneu)[k] = order[s][r ? HP - 1 - c : c];
  }
  for (int s = 0; s < 2; ++s) {  // slot counts per warp
    const int TPC = side_tpc(s), KM = side_km(HP, s), PPW = 32 / TPC;
    for (int w = tid; w < NPAIR / PPW; w += blockDim.x) {
      int k1 = 0, k2 = 0;
      for (int c = PPW * w; c < PPW * w + PPW; ++c) {
        k1 = max(k1, min(KM, (cnt[s][order[s][c]] + TPC - 1) / TPC));
        k2 = max(k2, min(KM, (cnt[s][order[s][HP - 1 - c]] + TPC - 1) / TPC));
      }
      (s ? tv.fk : tv.bk)[w] = k1 | (k2 << 8);
    }
  }
  // lists: a neuron's nonzero partners in round-robin order over the residues mod 8
  // (round k takes the k-th partner of every residue class, classes in order); each
  // partner's position follows from the class counts, so all entries are placed in
  // parallel
  constexpr uint64_t kClass0 = 0x0101010101010101ull;  // partners o with o % 8 == 0
  __shared__ int ccount[2][HP][8];
  for (int i = tid; i < 2 * HP * 8; i += blockDim.x) {
    const int s = i / (HP * 8), n = (i / 8) % HP, b = i % 8;
    ccount[s][n][b] = __popcll(nz[s][n] & (kClass0 << b));
  }
  __syncthreads();
  for (int i = tid; i < 2 * HP * HP; i += blockDim.x) {
    const int s = i / (HP * HP), n = (i / HP) % HP, o = i % HP;
    const uint64_t m = nz[s][n];
    if (!((m >> o) & 1ull)) continue;
    const int b = o & 7;
    const int k = __popcll(m & (kClass0 << b) & ((1ull << o) - 1ull));  // rank within its class
    int pos = 0;
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) {
      const int cb = ccount[s][n][bb];
      pos += min(cb, k) + ((bb < b && cb > k) ? 1 : 0);
    }
    if (!LTC_CHECKED_SKIP(pos < HP, 101)) lst[s][n][pos] = (unsigned char)o;
  }
  __syncthreads();
  // ... then every thread fills slots of both tables in parallel
  constexpr int NF = side_nt(HP, 1) * 2 * side_km(HP, 1), NB = side_nt(HP, 0) * 2 * side_km(HP, 0);
  for (int i = tid; i < NF + NB; i += blockDim.x) {
    const int s = i < NF ? 1 : 0;
    const int slot = s ? i : i - NF;
    const int TPC = side_tpc(s), KM = side_km(HP, s);
    const int j = slot % KM, r = (slot / KM) % 2, t = slot / (2 * KM);
    const int c = t / TPC, e = j * TPC + t % TPC;
    const int n = order[s][r ? HP - 1 - c : c];
    (s ? tv.fidx : tv.bidx)[slot] = e < min(cnt[s][n], TPC * KM) ? lst[s][n][e] : -1;
  }
}

// float4 stride (in float4 units) of a neuron's per-sample vector: odd, >= ns/4
__host__ __device__ inline int neuron_stride4(int ns) {
  const int s4 = (ns + 3) / 4;
  return (s4 & 1) ? s4 : s4 + 1;
}

// the warp's (K1, K2) -> the compile-time pass (K1 >= K2, both <= KM): one jump
// table on kw = K1 | K2 << 8, not a chain of compares
template <int V>
using IC = std::integral_constant<int, V>;
template <int KM, typename Fn>
__device__ __forceinline__ void dispatch_kk(int kw, Fn&& fn) {
  switch (kw) {
    case 0 | (0 << 8): if constexpr (KM >= 0) { fn(IC<0>{}, IC<0>{}); return; } break;
    case 1 | (0 << 8): if constexpr (KM >= 1) { fn(IC<1>{}, IC<0>{}); return; } break;
    case 1 | (1 << 8): if constexpr (KM >= 1) { fn(IC<1>{}, IC<1>{}); return; } break;
    case 2 | (0 << 8): if constexpr (KM >= 2) { fn(IC<2>{}, IC<0>{}); return; } break;
    case 2 | (1 << 8): if constexpr (KM >= 2) { fn(IC<2>{}, IC<1>{}); return; } break;
    case 2 | (2 << 8): if constexpr (KM >= 2) { fn(IC<2>{}, IC<2>{}); return; } break;
    case 3 | (0 << 8): if constexpr (KM >= 3) { fn(IC<3>{}, IC<0>{}); return; } break;
    case 3 | (1 << 8): if constexpr (KM >= 3) { fn(IC<3>{}, IC<1>{}); return; } break;
    case 3 | (2 << 8): if constexpr (KM >= 3) { fn(IC<3>{}, IC<2>{}); return; } break;
    case 3 | (3 << 8): if constexpr (KM >= 3) { fn(IC<3>{}, IC<3>{}); return; } break;
    case 4 | (0 << 8): if constexpr (KM >= 4) { fn(IC<4>{}, IC<0>{}); return; } break;
    case 4 | (1 << 8): if constexpr (KM >= 4) { fn(IC<4>{}, IC<1>{}); return; } break;
    case 4 | (2 << 8): if constexpr (KM >= 4) { fn(IC<4>{}, IC<2>{}); return; } break;
    case 4 | (3 << 8): if constexpr (KM >= 4) { fn(IC<4>{}, IC<3>{}); return; } break;
    case 4 | (4 << 8): if constexpr (KM >= 4) { fn(IC<4>{}, IC<4>{}); return; } break;
    case 5 | (0 << 8): if constexpr (KM >= 5) { fn(IC<5>{}, IC<0>{}); return; } break;
    case 5 | (1 << 8): if constexpr (KM >= 5) { fn(IC<5>{}, IC<1>{}); return; } break;
    case 5 | (2 << 8): if constexpr (KM >= 5) { fn(IC<5>{}, IC<2>{}); return; } break;
    case 5 | (3 << 8): if constexpr (KM >= 5) { fn(IC<5>{}, IC<3>{}); return; } break;
    case 5 | (4 << 8): if constexpr (KM >= 5) { fn(IC<5>{}, IC<4>{}); return; } break;
    case 5 | (5 << 8): if constexpr (KM >= 5) { fn(IC<5>{}, IC<5>{}); return; } break;
    case 6 | (0 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<0>{}); return; } break;
    case 6 | (1 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<1>{}); return; } break;
    case 6 | (2 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<2>{}); return; } break;
    case 6 | (3 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<3>{}); return; } break;
    case 6 | (4 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<4>{}); return; } break;
    case 6 | (5 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<5>{}); return; } break;
    case 6 | (6 << 8): if constexpr (KM >= 6) { fn(IC<6>{}, IC<6>{}); return; } break;
    default: break;
  }
  fn(IC<KM>{}, IC<KM>{});
}

// 16-bit byte offsets of a lane's slots (two per register)
template <int N>
struct Offsets {
  uint32_t w[(N + 1) / 2];
  __device__ __forceinline__ void set(int j, uint32_t o) {
    w[j / 2] = (j & 1) ? (w[j / 2] | (o << 16)) : o;
  }
  __device__ __forceinline__ uint32_t get(int j) const { return (j & 1) ? (w[j / 2] >> 16) : (w[j / 2] & 0xFFFFu); }
};

// ---- forward ------------------------------------------------------------------
// vbuf[2][HP][S] neuron-major states (S = 4 * neuron_stride4(ns)); snb/sdb [ns][LDV].
template <int HP>
struct SparseFwd {
  static constexpr int TPC = side_tpc(1), KM = side_km(HP, 1), NT = side_nt(HP, 1), LDV = HP + 4;
  float2 sl2[2][KM], nm2[2][KM], wp2[2][KM], we2[2][KM];  // duplicated constants
  Offsets<2 * KM> off;
  float cwe[2], cwp[2];

  template <int R, int K>
  __device__ __forceinline__ void row(const char* vb, float2 (&sn2)[2], float2 (&sd2)[2]) const {
    sn2[0] = sn2[1] = make_float2(cwe[R], cwe[R]);
    sd2[0] = sd2[1] = make_float2(cwp[R], cwp[R]);
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(vb + off.get(R * KM + j));
      const float2 th0 = tanh2(fma2(sl2[R][j], make_float2(v.x, v.y), nm2[R][j]));
      const float2 th1 = tanh2(fma2(sl2[R][j], make_float2(v.z, v.w), nm2[R][j]));
      sn2[0] = fma2(we2[R][j], th0, sn2[0]);
      sd2[0] = fma2(wp2[R][j], th0, sd2[0]);
      sn2[1] = fma2(we2[R][j], th1, sn2[1]);
      sd2[1] = fma2(wp2[R][j], th1, sd2[1]);
    }
  }

  // one block of 4 samples (vb = the block's first float4 in neuron 0's vector):
  // acc[0] = sum w_erev act, acc[1] = sum w_pos act per (r, i); the constant
  // halves of act = 1/2 + tanh/2 are in cwe/cwp, as in the dense kernel
  template <int K1, int K2>
  __device__ __forceinline__ void pass(const char* vb, float (&acc)[2][2 * kSB]) const {
    float2 sn2[2][2], sd2[2][2];
    row<0, K1>(vb, sn2[0], sd2[0]);
    row<1, K2>(vb, sn2[1], sd2[1]);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[0][r * kSB + 2 * h] = sn2[r][h].x;
        acc[0][r * kSB + 2 * h + 1] = sn2[r][h].y;
        acc[1][r * kSB + 2 * h] = sd2[r][h].x;
        acc[1][r * kSB + 2 * h + 1] = sd2[r][h].y;
      }
  }
};

template <int HP>
__global__ void __launch_bounds__(side_nt(HP, 1), 2) rec_fwd_sparse(RecFwdArgs a, SlotTablesView tv) {
  using F = SparseFwd<HP>;
  constexpr int NT = F::NT, KM = F::KM, LDV = F::LDV, TPC = F::TPC;
  using LR = LaneReduce<TPC, 2 * kSB>;
  extern __shared__ __align__(16) float smem[];
  const int ns = a.ns;
  const int S = 4 * neuron_stride4(ns);
  float* vbuf = smem;                 // [2][HP][S]
  float* snb2 = vbuf + 2 * HP * S;    // [2][ns][LDV]: step t in slot t & 1
  float* sdb2 = snb2 + 2 * ns * LDV;  // [2][ns][LDV]

  const int tid = threadIdx.x, lane = tid & 31, c = tid / TPC;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int b0 = blockIdx.x * ns;
  const int nvalid = min(ns, B - b0);
  const int nblk = (nvalid + kSB - 1) / kSB;
  const int kw = tv.fk[tid / 32];
  const bool overflow = *tv.overflow != 0;

  F f;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    f.cwe[r] = f.cwp[r] = 0.f;
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      const int base = (tid * 2 + r) * KM + j;
      int ix = tv.fidx[base];  // presynaptic neuron; the constants come from the dense pack
      if (LTC_CHECKED_SKIP(ix < HP && tv.fneu[2 * c + r] >= 0 && tv.fneu[2 * c + r] < HP, 102)) ix = -1;
      float4 pk = ix < 0 ? make_float4(0.f, 0.f, 0.f, 0.f) : a.pack[(long long)ix * HP + tv.fneu[2 * c + r]];
      pk.z *= 0.5f;
      pk.w *= 0.5f;
      f.sl2[r][j] = make_float2(pk.x, pk.x);
      f.nm2[r][j] = make_float2(pk.y, pk.y);
      f.wp2[r][j] = make_float2(pk.z, pk.z);
      f.we2[r][j] = make_float2(pk.w, pk.w);
      f.cwe[r] += pk.w;
      f.cwp[r] += pk.z;
      f.off.set(r * KM + j, (uint32_t)((ix < 0 ? 0 : ix) * S * 4));
    }
  }
  const int own = LR::own_base(lane);
  const int orow = own / kSB, osmp = own % kSB;
  const int q = tv.fneu[2 * c + orow];
  const float4 nq = a.nrn[q];
  const float cm = nq.x, cmgl = nq.x + nq.y, glvl = nq.w;
  const bool qvalid = q < H;
  const bool writer = LR::writer(lane);

  for (int i = tid; i < 2 * HP * S + 4 * ns * LDV; i += NT) smem[i] = 0.f;
  __syncthreads();
  if (a.h0) {
    for (int i = tid; i < nvalid * H; i += NT) {
      const int s = i / H, h = i % H;
      vbuf[h * S + s] = a.h0[(long long)(b0 + s) * H + h];
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
  int cur = 0;
  for (int t = 0; t < T; ++t) {
    __syncthreads();  // step t's sums visible; slot (t + 1) & 1 no longer read
    if (t + 1 < T) stage_sens(t + 1);
    const float* __restrict__ snb = snb2 + (t & 1) * ns * LDV;
    const float* __restrict__ sdb = sdb2 + (t & 1) * ns * LDV;
    for (int u = 0; u < U; ++u) {
      const long long n = (long long)t * U + u;
      const float* __restrict__ vc = vbuf + cur * HP * S;
      float* __restrict__ vn = vbuf + (cur ^ 1) * HP * S;
      for (int blk = 0; blk < nblk; ++blk) {
        float acc[2][2 * kSB];
        const char* vb = reinterpret_cast<const char*>(vc) + 16 * blk;
        dispatch_kk<KM>(kw, [&](auto K1, auto K2) {
          f.template pass<decltype(K1)::value, decltype(K2)::value>(vb, acc);
        });
        LR::template run<2>(acc, lane);
        const int s = blk * kSB + osmp;
        LTC_CHECK(s < S && q >= 0 && q < HP, 103);
        const float v = vc[q * S + s];
        const float wn = acc[0][0] + snb[s * LDV + q];
        const float wd = acc[1][0] + sdb[s * LDV + q];
        const float num = (cm * v + glvl) + wn;
        const float rr = rcp_approx((cmgl + wd) + a.eps);
        const float vnew = overflow ? __int_as_float(0x7fc00000) : num * rr;
        if (writer && qvalid && s < nvalid && !LTC_CHECKED_SKIP(b0 + s < B && q < H, 104)) {
          vn[q * S + s] = vnew;
          const long long bs = b0 + s;
          if (a.V) {
            a.V[(n * B + bs) * H + q] = v;
            a.R[(n * B + bs) * H + q] = rr;
          }
          if (u == U - 1 && a.out) a.out[(bs * T + t) * H + q] = vnew;
        }
      }
      __syncthreads();
      cur ^= 1;
    }
    cp_async_wait_all();
  }
  const float* vc = vbuf + cur * HP * S;
  for (int i = tid; i < nvalid * H; i += NT) {
    const int s = i / H, h = i % H;
    const long long bs = b0 + s;
    if (a.hT) a.hT[bs * H + h] = vc[h * S + s];
    if (a.V) a.V[((long long)T * U * B + bs) * H + h] = vc[h * S + s];
  }
}

// ---- backward -----------------------------------------------------------------
// AN/AD[2][HP][S] neuron-major adjoints (tanh space, a' = -a/4) of the unfold being
// processed and the next one; VS[3], RS[2], DIR, GSN, GSD [ns][LDV] as in the dense kernel.
template <int HP>
struct SparseBwd {
  static constexpr int TPC = side_tpc(0), KM = side_km(HP, 0), NT = side_nt(HP, 0), LDV = HP + 4;
  float2 sl2[2][KM], nm2[2][KM], wp2[2][KM], we2[2][KM];   // duplicated constants
  float2 Gwe[2][KM], Gwp[2][KM], Gdz[2][KM], Gdzv[2][KM];  // (even, odd) sample sums
  Offsets<2 * KM> off;

  // neuron R's K slots over one block; dv[h] = sum of dL/dz * (-sigma/2) for samples (2h, 2h+1)
  template <int R, int K>
  __device__ __forceinline__ void row(const char* an_b, const char* ad_b, const float4& vr, float2 (&dv)[2]) {
    const float2 m1 = make_float2(-1.f, -1.f);
    const float2 vp[2] = {make_float2(vr.x, vr.y), make_float2(vr.z, vr.w)};
    dv[0] = dv[1] = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const uint32_t o = off.get(R * KM + j);
      const float4 a4 = *reinterpret_cast<const float4*>(an_b + o);
      const float4 d4 = *reinterpret_cast<const float4*>(ad_b + o);
      const float2 an[2] = {make_float2(a4.x, a4.y), make_float2(a4.z, a4.w)};
      const float2 ad[2] = {make_float2(d4.x, d4.y), make_float2(d4.z, d4.w)};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // tanh space, as in the dense kernel: tn = tanh(-z/2), a' = -a/4
        const float2 tn = tanh2(fma2(sl2[R][j], vp[h], nm2[R][j]));
        const float2 dz = mul2(fma2(an[h], we2[R][j], mul2(ad[h], wp2[R][j])), fma2(tn, tn, m1));
        Gwe[R][j] = fma2(an[h], tn, Gwe[R][j]);
        Gwp[R][j] = fma2(ad[h], tn, Gwp[R][j]);
        Gdz[R][j] = add2(Gdz[R][j], dz);
        Gdzv[R][j] = fma2(dz, vp[h], Gdzv[R][j]);
        dv[h] = fma2(dz, sl2[R][j], dv[h]);
      }
    }
  }

  template <int K1, int K2>
  __device__ __forceinline__ void pass(const char* an_b, const char* ad_b, const float4 (&vr)[2],
                                       float (&acc)[1][2 * kSB]) {
    float2 dv[2][2];
    row<0, K1>(an_b, ad_b, vr[0], dv[0]);
    row<1, K2>(an_b, ad_b, vr[1], dv[1]);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[0][r * kSB + 2 * h] = dv[r][h].x;
        acc[0][r * kSB + 2 * h + 1] = dv[r][h].y;
      }
  }
};

template <int HP>
__global__ void __launch_bounds__(side_nt(HP, 0), 1) rec_bwd_sparse(RecBwdArgs a, SlotTablesView tv) {
  using F = SparseBwd<HP>;
  constexpr int NT = F::NT, KM = F::KM, LDV = F::LDV, kTPC = F::TPC;
  using LR = LaneReduce<kTPC, 2 * kSB>;
  extern __shared__ __align__(16) float smem[];
  const int ns = a.ns;
  const int S = 4 * neuron_stride4(ns);
  const int SL = ns * LDV;
  const int SA = HP * S;        // one neuron-major adjoint slab
  float* AN = smem;             // [2][SA]
  float* AD = AN + 2 * SA;      // [2][SA]
  float* VS = AD + 2 * SA;      // [3][SL]
  float* RS = VS + 3 * SL;      // [2][SL]
  float* DIR = RS + 2 * SL;
  float* GSN = DIR + SL;
  float* GSD = GSN + SL;
  float* GO = GSD + SL;         // [2][SL]
  float* red = GO + 2 * SL;     // [5][HP][kTPC]

  const int tid = threadIdx.x, lane = tid & 31, c = tid / kTPC, g = tid % kTPC;
  const int H = a.H, B = a.B, T = a.T, U = a.U;
  const int grp = blockIdx.x;
  const int b0 = grp * ns;
  const int nvalid = min(ns, B - b0);
  const int nblk = (nvalid + kSB - 1) / kSB;
  const int NTU = T * U;
  const int kw = tv.bk[tid / 32];
  const float bad = *tv.overflow ? __int_as_float(0x7fc00000) : 0.f;  // NaN poisons every output
  const int rowA = tv.bneu[2 * c], rowB = tv.bneu[2 * c + 1];

  F f;
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      const int base = (tid * 2 + r) * KM + j;
      int ix = tv.bidx[base];  // postsynaptic neuron; the constants come from the dense pack
      if (LTC_CHECKED_SKIP(ix < HP && rowA >= 0 && rowA < HP && rowB >= 0 && rowB < HP, 111)) ix = -1;
      float4 pk = ix < 0 ? make_float4(0.f, 0.f, 0.f, 0.f) : a.pack[(long long)(r ? rowB : rowA) * HP + ix];
      pk.x = -pk.x;  // negated half-scale constants: the gate argument is -z/2
      pk.y = -pk.y;
      f.sl2[r][j] = make_float2(pk.x, pk.x);
      f.nm2[r][j] = make_float2(pk.y, pk.y);
      f.wp2[r][j] = make_float2(pk.z, pk.z);
      f.we2[r][j] = make_float2(pk.w, pk.w);
      f.Gwe[r][j] = f.Gwp[r][j] = f.Gdz[r][j] = f.Gdzv[r][j] = make_float2(bad, bad);
      f.off.set(r * KM + j, (uint32_t)((ix < 0 ? 0 : ix) * S * 4));
    }
  const int own = LR::own_base(lane);
  const int orow = own / kSB, osmp = own % kSB;
  const int p = orow ? rowB : rowA;
  const float4 np_ = a.nrn[p];
  const float cm = np_.x, gl = np_.y, vl = np_.z;
  const bool pvalid = p < H;
  const bool writer = LR::writer(lane);
  float gcm = bad, ggl = bad, gvl = bad, san = bad, sad = bad;

  for (int i = tid; i < 4 * SA + 10 * SL; i += NT) smem[i] = 0.f;
  __syncthreads();

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
  __syncthreads();

  // per-neuron prep of unfold m for (sample s, neuron p), as in the dense kernel;
  // the adjoints go to the neuron-major slabs the synapse pass gathers from
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
    an_d[p * S + s] = -0.25f * an;
    ad_d[p * S + s] = -0.25f * ad;
  };

  if (writer && pvalid) {
    const int m = NTU - 1;
    for (int blk = 0; blk < nblk; ++blk) {
      const int s = blk * kSB + osmp;
      if (s < nvalid) {
        const long long bs = b0 + s;
        float gval = a.gout[bs * a.go_sb + (long long)(T - 1) * a.go_st + (long long)p * a.go_sh] + bad;
        if (a.gstate) gval += a.gstate[bs * H + p];
        prep(RS + (m % 2) * SL, VS + (m % 3) * SL, VS + ((m + 1) % 3) * SL, AN + (m % 2) * SA,
             AD + (m % 2) * SA, s, gval, true);
      }
    }
  }
  __syncthreads();

  int t = T - 1, k = U - 1;
  for (int n = NTU - 1; n >= 0; --n) {
    if (n >= 2) {
      stage_v(n - 2);
      stage_r(n - 2);
    }
    if (k == 0 && t >= 2) stage_go(t - 2);  // read at step t - 1's last unfold, >= 1 unfold later
    cp_async_commit();
    const int c2 = n % 2, c2m = c2 ^ 1;
    const int c3 = n % 3, c3m = (n + 2) % 3;
    const char* an_s = reinterpret_cast<const char*>(AN + c2 * SA);
    const char* ad_s = reinterpret_cast<const char*>(AD + c2 * SA);
    const float* vsn = VS + c3 * SL;
    const float* vsm = VS + c3m * SL;
    const float* rsm = RS + c2m * SL;
    float* an_m = AN + c2m * SA;
    float* ad_m = AD + c2m * SA;
    for (int blk = 0; blk < nblk; ++blk) {
      const float* vb = vsn + blk * kSB * LDV;
      const float4 vr[2] = {make_float4(vb[rowA], vb[LDV + rowA], vb[2 * LDV + rowA], vb[3 * LDV + rowA]),
                            make_float4(vb[rowB], vb[LDV + rowB], vb[2 * LDV + rowB], vb[3 * LDV + rowB])};
      float acc[1][2 * kSB];
      dispatch_kk<KM>(kw, [&](auto K1, auto K2) {
        f.template pass<decltype(K1)::value, decltype(K2)::value>(an_s + 16 * blk, ad_s + 16 * blk, vr, acc);
      });
      LR::template run<1>(acc, lane);
      const int s = blk * kSB + osmp;
      if (pvalid && writer && s < nvalid && !LTC_CHECKED_SKIP(s < ns && p < HP && b0 + s < B, 112)) {
        const int idx = s * LDV + p;
        float gval = fmaf(-2.0f, acc[0][0], DIR[idx]);
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
    cp_async_wait_all();
    __syncthreads();
    if (--k < 0) {
      k = U - 1;
      --t;
    }
  }

  // synapse partials at their dense positions (skipped synapses are never written)
  float* part = a.part + (long long)grp * 4 * HP * HP;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r ? rowB : rowA;
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      const int qi = tv.bidx[(tid * 2 + r) * KM + j];
      if (qi < 0 || LTC_CHECKED_SKIP(qi < HP && row >= 0 && row < HP, 113)) continue;
      const int idx = row * HP + qi;
      const float v0 = f.Gwe[r][j].x + f.Gwe[r][j].y, v1 = f.Gwp[r][j].x + f.Gwp[r][j].y;
      const float v2 = f.Gdz[r][j].x + f.Gdz[r][j].y, v3 = f.Gdzv[r][j].x + f.Gdzv[r][j].y;
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
  }
  // per-neuron sums, fixed order over the lanes of the pair
  for (int i = tid; i < 5 * HP * kTPC; i += NT) red[i] = 0.f;
  __syncthreads();
  if (writer) {
    red[(0 * HP + p) * kTPC + g] = gcm;
    red[(1 * HP + p) * kTPC + g] = ggl;
    red[(2 * HP + p) * kTPC + g] = gvl;
    red[(3 * HP + p) * kTPC + g] = san;
    red[(4 * HP + p) * kTPC + g] = sad;
  }
  __syncthreads();
  if (tid < HP) {
    float* pn = a.partn + (long long)grp * 5 * HP;
#pragma unroll
    for (int kk = 0; kk < 5; ++kk) {
      float sum = 0.f;
      for (int l = 0; l < kTPC; ++l) sum += red[(kk * HP + tid) * kTPC + l];
      pn[kk * HP + tid] = a.accumulate ? pn[kk * HP + tid] + sum : sum;
    }
  }
}


// ---- sensory backward over the nonzero sensory synapses -------------------------
// The sensory backward is the recurrent backward's synapse pass with the
// presynaptic neuron p replaced by the input d and no recurrence.  The (D, H) sensory
// pattern is cut into HP x HP blocks (HP = 32 for H <= 32, else 64; nqc column
// blocks); each block's slot tables (build_slots_kernel) give every lane its synapses,
// and a CTA = (block, row split) walks its rows in tiles of kSensRows.  With more than
// one column block, each writes its own dx partial, summed in a fixed order by the
// finish kernel.  Per tile, g_sn / g_sd are staged
// neuron-major (column q, rows) exactly as the recurrent adjoints, and x row-major as
// the recurrent states; the 4 gradient sums per synapse stay in registers over the
// whole row split, dx[row][d] comes out of the lane reduction.  Tanh space as in the
// dense sensory backward: the -1/4 of a' = -g/4 is folded into the weights, so the
// raw g_sn / g_sd are staged and the A_n / A_d sums are scaled by -1/4 at the end.
constexpr int kSensRows = 64;

template <int HP>
__global__ void __launch_bounds__(side_nt(HP, 0), 1)
    sens_bwd_sparse(SensBwdArgs a, SlotTablesView tv, size_t chunk_bytes, long long rows_per_split, int nqc,
                    float* dxpart) {
  using F = SparseBwd<HP>;
  constexpr int NT = F::NT, KM = F::KM, LDV = F::LDV, kTPC = F::TPC, R = kSensRows;
  using LR = LaneReduce<kTPC, 2 * kSB>;
  extern __shared__ __align__(16) float smem[];
  const int S = 4 * neuron_stride4(R);
  float* GN = smem;              // [2][HP][S]  g_sn, neuron-major
  float* GD = GN + 2 * HP * S;   // [2][HP][S]  g_sd
  float* XS = GD + 2 * HP * S;   // [2][R][LDV] x of the chunk's inputs
  const int chunk = blockIdx.x, split = blockIdx.y;
  {  // this chunk's tables
    const size_t o = (size_t)chunk * chunk_bytes;
    tv.bneu = reinterpret_cast<int*>(reinterpret_cast<char*>(tv.bneu) + o);
    tv.bk = reinterpret_cast<int*>(reinterpret_cast<char*>(tv.bk) + o);
    tv.bidx = reinterpret_cast<int*>(reinterpret_cast<char*>(tv.bidx) + o);
    tv.overflow = reinterpret_cast<int*>(reinterpret_cast<char*>(tv.overflow) + o);
  }
  const int d0 = (chunk / nqc) * HP, q0 = (chunk % nqc) * HP;
  const int tid = threadIdx.x, lane = tid & 31, c = tid / kTPC;
  const int D = a.D, H = a.H;
  const int kw = tv.bk[tid / 32];
  const float bad = *tv.overflow ? __int_as_float(0x7fc00000) : 0.f;  // NaN poisons every output
  const int rowA = tv.bneu[2 * c], rowB = tv.bneu[2 * c + 1];

  F f;
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      const int base = (tid * 2 + r) * KM + j;
      int ix = tv.bidx[base];  // column q
      if (LTC_CHECKED_SKIP(ix < HP && rowA >= 0 && rowA < HP && rowB >= 0 && rowB < HP, 121)) ix = -1;
      const int d = d0 + (r ? rowB : rowA);
      float4 pk = (ix < 0 || d >= D) ? make_float4(0.f, 0.f, 0.f, 0.f) : a.spack[(long long)d * a.HP + q0 + ix];
      pk.x = -pk.x;  // gate argument -z/2
      pk.y = -pk.y;
      pk.z *= -0.25f;  // a' = -g/4 folded into the weights
      pk.w *= -0.25f;
      f.sl2[r][j] = make_float2(pk.x, pk.x);
      f.nm2[r][j] = make_float2(pk.y, pk.y);
      f.wp2[r][j] = make_float2(pk.z, pk.z);
      f.we2[r][j] = make_float2(pk.w, pk.w);
      f.Gwe[r][j] = f.Gwp[r][j] = f.Gdz[r][j] = f.Gdzv[r][j] = make_float2(bad, bad);
      f.off.set(r * KM + j, (uint32_t)((ix < 0 ? 0 : ix) * S * 4));
    }
  const int own = LR::own_base(lane);
  const int orow = own / kSB, osmp = own % kSB;
  const int p = orow ? rowB : rowA;
  const bool pvalid = d0 + p < D;
  const bool writer = LR::writer(lane);
  const long long r_begin = split * rows_per_split;
  const long long r_end = min(a.rows, r_begin + rows_per_split);

  auto stage = [&](long long rt, int buf) {
    const int nr = (int)min((long long)R, r_end - rt);
    float* gn = GN + buf * HP * S;
    float* gd = GD + buf * HP * S;
    float* xs = XS + buf * R * LDV;
    for (int i = tid; i < R * HP; i += NT) {
      const int r = i / HP, q = i % HP;  // consecutive threads read consecutive columns of a row
      const bool ok = r < nr && q0 + q < H;
      const long long src = ok ? (rt + r) * H + q0 + q : 0;
      cp_async4_zfill(gn + q * S + r, a.gsn + src, ok);
      cp_async4_zfill(gd + q * S + r, a.gsd + src, ok);
      const bool okx = r < nr && d0 + q < D;
      cp_async4_zfill(xs + r * LDV + q, a.x + (okx ? (rt + r) * D + d0 + q : 0), okx);
    }
    cp_async_commit();
  };
  if (r_begin < r_end) stage(r_begin, 0);
  int buf = 0;
  for (long long rt = r_begin; rt < r_end; rt += R, buf ^= 1) {
    const int nr = (int)min((long long)R, r_end - rt);
    cp_async_wait_all();
    __syncthreads();  // tile rt landed; the other buffer is free again
    if (rt + R < r_end) stage(rt + R, buf ^ 1);
    const char* an_s = reinterpret_cast<const char*>(GN + buf * HP * S);
    const char* ad_s = reinterpret_cast<const char*>(GD + buf * HP * S);
    const float* xs = XS + buf * R * LDV;
    const int nblk = (nr + kSB - 1) / kSB;
    for (int blk = 0; blk < nblk; ++blk) {
      const float* vb = xs + blk * kSB * LDV;
      const float4 vr[2] = {make_float4(vb[rowA], vb[LDV + rowA], vb[2 * LDV + rowA], vb[3 * LDV + rowA]),
                            make_float4(vb[rowB], vb[LDV + rowB], vb[2 * LDV + rowB], vb[3 * LDV + rowB])};
      float acc[1][2 * kSB];
      dispatch_kk<KM>(kw, [&](auto K1, auto K2) {
        f.template pass<decltype(K1)::value, decltype(K2)::value>(an_s + 16 * blk, ad_s + 16 * blk, vr, acc);
      });
      LR::template run<1>(acc, lane);
      const int s = blk * kSB + osmp;
      if (writer && pvalid && s < nr) {
        const float v = -2.0f * acc[0][0] + bad;  // sl holds -sigma/2
        const long long o = (rt + s) * D + d0 + p;
        if (LTC_CHECKED_SKIP(rt + s < a.rows && d0 + p < D, 122)) continue;
        if (nqc == 1) a.dx[o] = v;
        else dxpart[(long long)(chunk % nqc) * a.rows * D + o] = v;
      }
    }
  }
  // synapse partials at their dense positions (skipped synapses are never written)
  const long long slab = (long long)D * a.HP;
  float* part = a.part + (long long)split * 4 * slab;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int d = d0 + (r ? rowB : rowA);
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      const int qi = tv.bidx[(tid * 2 + r) * KM + j];
      if (qi < 0 || d >= D || LTC_CHECKED_SKIP(qi < HP && q0 + qi < a.HP, 123)) continue;
      const long long idx = (long long)d * a.HP + q0 + qi;
      part[idx] = -0.25f * (f.Gwe[r][j].x + f.Gwe[r][j].y);
      part[slab + idx] = -0.25f * (f.Gwp[r][j].x + f.Gwp[r][j].y);
      part[2 * slab + idx] = f.Gdz[r][j].x + f.Gdz[r][j].y;
      part[3 * slab + idx] = f.Gdzv[r][j].x + f.Gdzv[r][j].y;
    }
  }
}


template <typename K, typename Args>
cudaError_t launch_plain(K kernel, const Args& a, const SlotTablesView& tv, int grid, int threads, size_t smem,
                         cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kernel<<<grid, threads, smem, st>>>(a, tv);
  return cudaGetLastError();
}

}  // namespace

size_t sparse_tables_bytes(int HP) {
  if (HP > 64) return csp_tables_bytes(HP);
  size_t at[7];
  return tables_layout(HP, at);
}


void plan_sparse(RecPlan& p, int B, int num_sms) {
  const int HP = p.HP;  // 32 or 64
  const int LDV = HP + 4;
  const int blocks = (B + kSB - 1) / kSB;
  const size_t smem_cap = 227 * 1024 - 1024;
  // backward: 4 neuron-major adjoint slabs + 10 [ns][LDV] slabs + the reduction area
  auto bwd_bytes = [&](int ns) {
    const int S = 4 * neuron_stride4(ns);
    return ((size_t)4 * HP * S + 10 * (size_t)ns * LDV + 5 * HP * side_tpc(0)) * sizeof(float);
  };
  int cap = 1;
  while (bwd_bytes((cap + 1) * kSB) <= smem_cap) ++cap;
  // blocks per CTA: as many waves as the cap forces, spread evenly over them
  const long long per_wave = (long long)num_sms * cap;
  const long long waves = (blocks + per_wave - 1) / per_wave;
  int per = (int)((blocks + waves * num_sms - 1) / (waves * num_sms));
  if (per > cap) per = cap;
  if (per < 1) per = 1;
  const int ns = per * kSB;
  const int S = 4 * neuron_stride4(ns);
  // the forward (128 registers, small shared memory) runs two CTAs per SM: its groups
  // are planned over twice the SMs, so two groups overlap their per-unfold latency
  const int per_f = (int)((blocks + 2LL * num_sms - 1) / (2LL * num_sms));
  const int ns_f = per_f * kSB;
  const int S_f = 4 * neuron_stride4(ns_f);
  p.sparse = true;
  p.ns_fwd = ns_f;
  p.ns_bwd = ns;
  p.grid_fwd = (B + ns_f - 1) / ns_f;
  p.grid_bwd = (B + ns - 1) / ns;
  p.threads_fwd = side_nt(HP, 1);
  p.threads_bwd = side_nt(HP, 0);
  p.slots_bwd = p.grid_bwd;
  p.smem_fwd = ((size_t)2 * HP * S_f + 4 * (size_t)ns_f * LDV) * sizeof(float);
  p.smem_bwd = bwd_bytes(ns);
  p.tanh_space = true;
}


// ---- sensory backward (skipped sensory synapses) ---------------------------------
// block width of the sensory backward's slot tables: 32 for HP = 32, else 64
static inline int sens_bh(int HP) { return HP == 32 ? 32 : 64; }

static inline void sens_blocks(int D, int H, int HP, int* ndc, int* nqc) {
  const int bh = sens_bh(HP);
  *ndc = (D + bh - 1) / bh;
  *nqc = (H + bh - 1) / bh;
}

size_t sens_bwd_tables_bytes(int D, int H, int HP) {
  int ndc, nqc;
  sens_blocks(D, H, HP, &ndc, &nqc);
  size_t at[7];
  return (size_t)ndc * nqc * tables_layout(sens_bh(HP), at);
}

void plan_sensory_bwd_sparse(SensBwdPlan& p, long long rows, int D, int H, int HP, int num_sms) {
  int ndc, nqc;
  sens_blocks(D, H, HP, &ndc, &nqc);
  int ns = num_sms / (ndc * nqc);
  if (ns < 1) ns = 1;
  const long long max_split = (rows + kSensRows - 1) / kSensRows;
  if (ns > max_split) ns = (int)(max_split > 0 ? max_split : 1);
  p.qc = sens_bh(HP);
  p.nqc = nqc;
  p.dpc = sens_bh(HP);
  p.ndc = ndc;
  p.nsplit = ns;
  p.part_floats = (size_t)ns * 4 * D * HP;
  p.dxpart_floats = nqc > 1 ? (size_t)nqc * rows * D : 0;
}

cudaError_t launch_build_sens_slots(const PackArgs& pa, void* tables, cudaStream_t st) {
  int ndc, nqc;
  sens_blocks(pa.D, pa.H, pa.HP, &ndc, &nqc);
  const int bh = sens_bh(pa.HP);
  size_t at[7];
  const size_t cb = tables_layout(bh, at);
  const SlotTablesView tv = tables_view(tables, bh);
  if (bh == 64)
    build_slots_kernel<64><<<ndc * nqc, 256, 0, st>>>(tv, pa.sw, pa.sw, pa.H, pa.D, pa.H, nqc, cb);
  else
    build_slots_kernel<32><<<ndc * nqc, 256, 0, st>>>(tv, pa.sw, pa.sw, pa.H, pa.D, pa.H, nqc, cb);
  return cudaGetLastError();
}

cudaError_t launch_sensory_bwd_sparse(const SensBwdArgs& a, const SensBwdPlan& p, const void* tables,
                                      float* dxpart, cudaStream_t st) {
  if (a.rows <= 0) return cudaSuccess;
  long long rps = (a.rows + p.nsplit - 1) / p.nsplit;
  rps = (rps + kSensRows - 1) / kSensRows * kSensRows;
  const int bh = sens_bh(a.HP);
  size_t at[7];
  const size_t cb = tables_layout(bh, at);
  const SlotTablesView tv = tables_view(const_cast<void*>(tables), bh);
  const int S = 4 * neuron_stride4(kSensRows);
  const size_t smem = ((size_t)4 * bh * S + (size_t)2 * kSensRows * (bh + 4)) * sizeof(float);
  const dim3 grid(p.ndc * p.nqc, p.nsplit);
  cudaError_t e;
  if (bh == 64) {
    e = cudaFuncSetAttribute(sens_bwd_sparse<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sens_bwd_sparse<64><<<grid, side_nt(64, 0), smem, st>>>(a, tv, cb, rps, p.nqc, dxpart);
  } else {
    e = cudaFuncSetAttribute(sens_bwd_sparse<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sens_bwd_sparse<32><<<grid, side_nt(32, 0), smem, st>>>(a, tv, cb, rps, p.nqc, dxpart);
  }
  return cudaGetLastError();
}

cudaError_t launch_build_slots(const PackArgs& pa, void* tables, cudaStream_t st) {
  if (pa.HP > 64) return launch_build_csp(pa, tables, st);
  const SlotTablesView tv = tables_view(tables, pa.HP);
  if (pa.HP == 64)
    build_slots_kernel<64><<<1, 256, 0, st>>>(tv, pa.w_pos, pa.w_erev, pa.H, pa.H, pa.H, 1, 0);
  else
    build_slots_kernel<32><<<1, 256, 0, st>>>(tv, pa.w_pos, pa.w_erev, pa.H, pa.H, pa.H, 1, 0);
  return cudaGetLastError();
}

cudaError_t launch_sparse_fwd(const RecFwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st) {
  if (p.streamed) return launch_csp_fwd(a, p, tables, st);
  const SlotTablesView tv = tables_view(const_cast<void*>(tables), p.HP);
  return p.HP == 64 ? launch_plain(rec_fwd_sparse<64>, a, tv, p.grid_fwd, p.threads_fwd, p.smem_fwd, st)
                    : launch_plain(rec_fwd_sparse<32>, a, tv, p.grid_fwd, p.threads_fwd, p.smem_fwd, st);
}

cudaError_t launch_sparse_bwd(const RecBwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st) {
  if (p.streamed) return launch_csp_bwd(a, p, tables, st);
  const SlotTablesView tv = tables_view(const_cast<void*>(tables), p.HP);
  return p.HP == 64 ? launch_plain(rec_bwd_sparse<64>, a, tv, p.grid_bwd, p.threads_bwd, p.smem_bwd, st)
                    : launch_plain(rec_bwd_sparse<32>, a, tv, p.grid_bwd, p.threads_bwd, p.smem_bwd, st);
}

}  // namespace ltc
