// Sensory conductance pass, forward and backward, batched over all B*T rows.
//
// The sensory term  sn[q] = sum_d sw*serev*act,  sd[q] = sum_d sw*act,
// act = sigmoid(ssig*(x[d]-smu)), does not depend on the state, so it is
// computed for every (b,t) row in one launch before the recurrence
// (row = b*T + t, x is (rows, D)).
//
// Forward: thread = (column q, row group rg), RB rows per thread, no
//   cross-thread reduction; the gate pack of a chunk of DC inputs and the x
//   tile are staged in shared memory and shared by the row groups.
// Backward: thread = (2 inputs d, lane group g) owning 8 columns of a QC-column
//   chunk (the same map as the recurrent backward kernel with p -> d); it
//   accumulates the 4 synapse-gradient sums in registers over all rows of its
//   row split and writes them once; dx[row][d] is reduced over the TPC lanes.
#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace ltc {

namespace {

constexpr int kRB = 8;  // rows per thread (forward)
constexpr int kSB = 4;  // rows per register block (backward)
constexpr int kRT = 32; // rows per staged tile (backward)

struct SensFwdGeom {
  int HPW, RG, NT, TR, DC;
};

__host__ __device__ inline SensFwdGeom sens_fwd_geom(int HPW, int D) {
  SensFwdGeom g;
  g.HPW = HPW;
  g.RG = 512 / HPW;
  g.NT = HPW * g.RG;
  g.TR = g.RG * kRB;
  int dc = 4096 / HPW;
  if (dc < 4) dc = 4;
  if (dc > D) dc = D;
  g.DC = dc;
  return g;
}

__global__ void __launch_bounds__(512, 2) sens_fwd_kernel(SensFwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  const SensFwdGeom G = sens_fwd_geom(a.HP, a.D);
  float4* pks = reinterpret_cast<float4*>(smem);  // [DC][HPW]
  float* xs = smem + 4 * G.DC * G.HPW;           // [DC][TR]
  const int tid = threadIdx.x;
  const int q = tid % G.HPW, rg = tid / G.HPW;
  const int H = a.H, D = a.D;
  const long long ntiles = (a.rows + G.TR - 1) / G.TR;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long row0 = tile * G.TR;
    // act = 0.5 + 0.5*tanh(z/2): accumulate sum w*tanh, add sum w at the end
    float sn[kRB], sd[kRB], csw = 0.f, cswe = 0.f;
#pragma unroll
    for (int r = 0; r < kRB; ++r) sn[r] = sd[r] = 0.f;
    for (int d0 = 0; d0 < D; d0 += G.DC) {
      const int dc = min(G.DC, D - d0);
      __syncthreads();
      for (int i = tid; i < dc * G.HPW; i += blockDim.x) pks[i] = a.spack[(long long)d0 * G.HPW + i];
      for (int i = tid; i < G.TR * dc; i += blockDim.x) {
        const int r = i / dc, dd = i % dc;
        const long long row = row0 + r;
        xs[dd * G.TR + r] = row < a.rows ? a.x[row * D + d0 + dd] : 0.f;
      }
      __syncthreads();
      const float* xr = xs + rg * kRB;
      for (int dd = 0; dd < dc; ++dd) {
        const float4 w = pks[dd * G.HPW + q];
        cswe += w.w;
        csw += w.z;
        const float4 x0 = *reinterpret_cast<const float4*>(xr + dd * G.TR);
        const float4 x1 = *reinterpret_cast<const float4*>(xr + dd * G.TR + 4);
        const float xv[kRB] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int r = 0; r < kRB; ++r) {
          const float th = tanh_approx(fmaf(w.x, xv[r], w.y));
          sn[r] = fmaf(w.w, th, sn[r]);
          sd[r] = fmaf(w.z, th, sd[r]);
        }
      }
    }
    if (q < H) {
#pragma unroll
      for (int r = 0; r < kRB; ++r) {
        const long long row = row0 + rg * kRB + r;
        if (row < a.rows) {
          a.sn[row * H + q] = 0.5f * (cswe + sn[r]);
          a.sd[row * H + q] = 0.5f * (csw + sd[r]);
        }
      }
    }
  }
}

// Resident variant for small sensory matrices (D*HPW float4 <= kResidentBytes): the
// whole gate pack stays in shared memory for the kernel's lifetime, the per-column
// weight sums are computed once, and the x tiles ([d][row], transposed) are
// double-buffered with cp.async so their loads overlap the previous tile's gates.
constexpr size_t kResidentBytes = 144 * 1024;

template <int HPW>
__global__ void __launch_bounds__(512, 1) sens_fwd_resident(SensFwdArgs a) {
  constexpr int RG = 512 / HPW, TR = RG * kRB;
  extern __shared__ __align__(16) float smem[];
  const int D = a.D, H = a.H;
  float4* pks = reinterpret_cast<float4*>(smem);  // [D][HPW]
  float* xs = smem + 4 * D * HPW;                 // [2][D][TR]
  const int tid = threadIdx.x;
  const int q = tid % HPW, rg = tid / HPW;
  const long long ntiles = (a.rows + TR - 1) / TR;

  auto stage_x = [&](long long tile, int buf) {
    float* dst = xs + buf * D * TR;
    const long long row0 = tile * TR;
    for (int i = tid; i < TR * D; i += 512) {
      const int r = i % TR, d = i / TR;  // consecutive lanes -> consecutive rows: conflict-free stores
      const long long row = row0 + r;
      if (row < a.rows) cp_async4(dst + d * TR + r, a.x + row * D + d);
      else dst[d * TR + r] = 0.f;
    }
    cp_async_commit();
  };
  for (int i = tid; i < D * HPW; i += 512) cp_async16(pks + i, a.spack + i);
  long long tile = blockIdx.x;
  if (tile < ntiles) stage_x(tile, 0);
  cp_async_wait_all();
  __syncthreads();
  float cswe = 0.f, csw = 0.f;  // act = 0.5 + 0.5 tanh: sum_d w / 2 is added at the end
  for (int d = 0; d < D; ++d) {
    const float4 w = pks[d * HPW + q];
    cswe += w.w;
    csw += w.z;
  }
  int buf = 0;
  for (; tile < ntiles; tile += gridDim.x, buf ^= 1) {
    if (tile + gridDim.x < ntiles) stage_x(tile + gridDim.x, buf ^ 1);
    float sn[kRB], sd[kRB];
#pragma unroll
    for (int r = 0; r < kRB; ++r) sn[r] = sd[r] = 0.f;
    const float* xr = xs + buf * D * TR + rg * kRB;
#pragma unroll 2
    for (int d = 0; d < D; ++d) {
      const float4 w = pks[d * HPW + q];
      const float4 x0 = *reinterpret_cast<const float4*>(xr + d * TR);
      const float4 x1 = *reinterpret_cast<const float4*>(xr + d * TR + 4);
      const float xv[kRB] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int r = 0; r < kRB; ++r) {
        const float th = tanh_approx(fmaf(w.x, xv[r], w.y));
        sn[r] = fmaf(w.w, th, sn[r]);
        sd[r] = fmaf(w.z, th, sd[r]);
      }
    }
    if (q < H) {
#pragma unroll
      for (int r = 0; r < kRB; ++r) {
        const long long row = tile * TR + rg * kRB + r;
        if (row < a.rows) {
          a.sn[row * H + q] = 0.5f * (cswe + sn[r]);
          a.sd[row * H + q] = 0.5f * (csw + sd[r]);
        }
      }
    }
    cp_async_wait_all();
    __syncthreads();
  }
}

template <int QC>
struct SensBwdGeom {
  static constexpr int NT = 256;         // threads
  static constexpr int TPC = QC / 8;     // lanes sharing an input pair
  static constexpr int NGD = NT / TPC;   // input groups; each thread owns 2 inputs
  static constexpr int DPC = 2 * NGD;    // inputs per CTA (= 4096 / QC)
  static constexpr int LDG = QC + 4;
  __device__ __forceinline__ static int sub(int j, int g) { return (j / 4) * (QC / 2) + 4 * g + (j % 4); }
};

// Thread = (input pair c, lane g): inputs d_r = d0 + c + r*NGD (r < 2), columns
// q0 + sub(j, g).  The per-row adjoint loads (8 columns of gsn, gsd) are shared
// by the two inputs.
// TS (tanh space): the recurrent backward also produced the column sums of g_sn,
// g_sd (= sum of a_n, a_d); the gate is evaluated as tn = tanh(-z/2) = -t, with
// a' = -g/4 the finish kernel adds the g/2 part of sum g*act:
//   dL/dz = (a'_n swe + a'_d sw)(tn^2 - 1),  g act = g/2 + 2 a' tn.
// The -1/4 is folded into the weight registers (dz) and into the final scale of
// the An/Ad sums, so the adjoint tiles are staged raw.
// Tiles of kRT rows (gsn, gsd, x) are double-buffered with cp.async (zero-filled
// outside the valid rows/columns), so the next tile's loads overlap this one's math.
template <int QC, bool TS>
__global__ void __launch_bounds__(256, 1) sens_bwd_kernel(SensBwdArgs a, int nqc, long long rows_per_split,
                                                          float* dxpart) {
  using G = SensBwdGeom<QC>;
  constexpr int TPC = G::TPC, DPC = G::DPC, LDG = G::LDG, NT = G::NT, NGD = G::NGD;
  constexpr int NI = 2 * kSB;
  using LR = LaneReduce<TPC, NI>;
  extern __shared__ __align__(16) float smem[];
  constexpr int TILE = 2 * kRT * LDG + kRT * DPC;  // floats of one buffer
  // buffer b: GN [kRT][LDG], GD [kRT][LDG], XS [kRT][DPC] at smem + b*TILE

  const int tid = threadIdx.x, lane = tid & 31;
  const int c = tid / TPC, g = tid % TPC;
  const int dchunk = blockIdx.x / nqc, qc = blockIdx.x % nqc;
  const int d0 = dchunk * DPC, q0 = qc * QC;
  const int D = a.D, H = a.H, HP = a.HP;

  float sl[2][8], nm[2][8], sw[2][8], swe[2][8];
  float An[2][8], Ad[2][8], Dz[2][8], Dzx[2][8];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = d0 + c + r * NGD;
      float4 pk = make_float4(0.f, 0.f, 0.f, 0.f);
      if (d < D) pk = a.spack[(long long)d * HP + q0 + G::sub(j, g)];
      sl[r][j] = TS ? -pk.x : pk.x; nm[r][j] = TS ? -pk.y : pk.y;
      sw[r][j] = TS ? -0.25f * pk.z : pk.z; swe[r][j] = TS ? -0.25f * pk.w : pk.w;
      An[r][j] = Ad[r][j] = Dz[r][j] = Dzx[r][j] = 0.f;
    }
  const int own = LR::own_base(lane);
  const bool writer = LR::writer(lane);
  const int hq = min(QC, H - q0);  // valid columns of this chunk
  const long long r_begin = blockIdx.y * rows_per_split;
  const long long r_end = min(a.rows, r_begin + rows_per_split);
  const long long ndx = a.rows * D;

  auto stage = [&](long long rt, int buf) {
    const int nr = (int)min((long long)kRT, r_end - rt);
    float* GN = smem + buf * TILE;
    float* GD = GN + kRT * LDG;
    float* XS = GD + kRT * LDG;
    for (int i = tid; i < kRT * QC; i += NT) {
      const int r = i / QC, cc = i % QC;
      const bool ok = r < nr && cc < hq;
      const long long src = ok ? (rt + r) * H + q0 + cc : 0;
      cp_async4_zfill(GN + r * LDG + cc, a.gsn + src, ok);
      cp_async4_zfill(GD + r * LDG + cc, a.gsd + src, ok);
    }
    for (int i = tid; i < kRT * DPC; i += NT) {
      const int r = i / DPC, cc = i % DPC;
      const bool ok = r < nr && d0 + cc < D;
      cp_async4_zfill(XS + i, a.x + (ok ? (rt + r) * D + d0 + cc : 0), ok);
    }
    cp_async_commit();
  };
  if (r_begin < r_end) stage(r_begin, 0);
  int buf = 0;
  for (long long rt = r_begin; rt < r_end; rt += kRT, buf ^= 1) {
    const int nr = (int)min((long long)kRT, r_end - rt);
    cp_async_wait_all();
    __syncthreads();  // tile rt landed; the other buffer is free again
    if (rt + kRT < r_end) stage(rt + kRT, buf ^ 1);
    const float* GN = smem + buf * TILE;
    const float* GD = GN + kRT * LDG;
    const float* XS = GD + kRT * LDG;
    const int nblk = (nr + kSB - 1) / kSB;
    for (int blk = 0; blk < nblk; ++blk) {
      float acc[1][NI];
#pragma unroll
      for (int i = 0; i < kSB; ++i) {
        const int row = blk * kSB + i;
        const float* ar = GN + row * LDG + 4 * g;
        const float* dr = GD + row * LDG + 4 * g;
        const float4 a0 = *reinterpret_cast<const float4*>(ar);
        const float4 a1 = *reinterpret_cast<const float4*>(ar + QC / 2);
        const float4 e0 = *reinterpret_cast<const float4*>(dr);
        const float4 e1 = *reinterpret_cast<const float4*>(dr + QC / 2);
        const float an8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float ad8[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float xv = XS[row * DPC + c + r * NGD];
          if constexpr (TS) {
            // synapses j, j+1 as packed f32x2 pairs
            const float2 x2 = make_float2(xv, xv), m1 = make_float2(-1.f, -1.f);
            float2 dxs = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int j = 2 * k;
              const float2 sl2 = make_float2(sl[r][j], sl[r][j + 1]), nm2 = make_float2(nm[r][j], nm[r][j + 1]);
              const float2 an2 = make_float2(an8[j], an8[j + 1]), ad2 = make_float2(ad8[j], ad8[j + 1]);
              const float2 tn = tanh2(fma2(sl2, x2, nm2));
              const float2 dz = mul2(fma2(an2, make_float2(swe[r][j], swe[r][j + 1]),
                                          mul2(ad2, make_float2(sw[r][j], sw[r][j + 1]))),
                                     fma2(tn, tn, m1));
              float2 t;
              t = fma2(an2, tn, make_float2(An[r][j], An[r][j + 1])); An[r][j] = t.x; An[r][j + 1] = t.y;
              t = fma2(ad2, tn, make_float2(Ad[r][j], Ad[r][j + 1])); Ad[r][j] = t.x; Ad[r][j + 1] = t.y;
              t = add2(dz, make_float2(Dz[r][j], Dz[r][j + 1])); Dz[r][j] = t.x; Dz[r][j + 1] = t.y;
              t = fma2(dz, x2, make_float2(Dzx[r][j], Dzx[r][j + 1])); Dzx[r][j] = t.x; Dzx[r][j + 1] = t.y;
              dxs = fma2(dz, sl2, dxs);
            }
            acc[0][r * kSB + i] = dxs.x + dxs.y;
          } else {
            float dxs = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float act = gate_tanh(sl[r][j], nm[r][j], xv);
              const float sp = fmaf(-act, act, act);
              const float dz = fmaf(an8[j], swe[r][j], ad8[j] * sw[r][j]) * sp;
              An[r][j] = fmaf(an8[j], act, An[r][j]);
              Ad[r][j] = fmaf(ad8[j], act, Ad[r][j]);
              Dz[r][j] += dz;
              Dzx[r][j] = fmaf(dz, xv, Dzx[r][j]);
              dxs = fmaf(dz, sl[r][j], dxs);
            }
            acc[0][r * kSB + i] = dxs;
          }
        }
      }
      LR::template run<1>(acc, lane);
      if (writer) {
#pragma unroll
        for (int o = 0; o < LR::OWN; ++o) {
          const int item = own + o;
          const int row = blk * kSB + item % kSB;
          const int d = d0 + c + (item / kSB) * NGD;
          if (row < nr && d < D) {
            const float v = (TS ? -2.0f : 2.0f) * acc[0][o];  // sl holds (-)sigma/2
            const long long idx = (rt + row) * D + d;
            if (nqc == 1) a.dx[idx] = v;
            else dxpart[qc * ndx + idx] = v;
          }
        }
      }
    }
  }
  const long long slab = (long long)D * HP;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int d = d0 + c + r * NGD;
    if (d >= D) continue;
    float* part = a.part + (long long)blockIdx.y * 4 * slab + (long long)d * HP + q0;
    const float sc = TS ? -0.25f : 1.0f;  // An/Ad were summed with the raw adjoints
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int cc = G::sub(j, g);
      part[cc] = sc * An[r][j];
      part[slab + cc] = sc * Ad[r][j];
      part[2 * slab + cc] = Dz[r][j];
      part[3 * slab + cc] = Dzx[r][j];
    }
  }
}

int pick_qc(int HP) {
  for (int qc = 256; qc >= 32; qc >>= 1)
    if (HP % qc == 0) return qc;
  return 32;
}

}  // namespace

cudaError_t launch_sensory_fwd(const SensFwdArgs& a, int num_sms, cudaStream_t st) {
  if (a.rows <= 0) return cudaSuccess;
  const int TRr = (512 / (a.HP > 0 ? a.HP : 1)) * kRB;
  const size_t smem_res = (size_t)a.D * a.HP * 16 + (size_t)2 * a.D * TRr * 4;
  if ((a.HP == 32 || a.HP == 64) && (size_t)a.D * a.HP * 16 <= kResidentBytes && smem_res <= 220 * 1024) {
    const int TR = TRr;
    const size_t smem = smem_res;
    const long long ntiles = (a.rows + TR - 1) / TR;
    const int grid = (int)(ntiles < num_sms ? ntiles : num_sms);
    cudaError_t e;
    if (a.HP == 64) {
      e = cudaFuncSetAttribute(sens_fwd_resident<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      sens_fwd_resident<64><<<grid, 512, smem, st>>>(a);
    } else {
      e = cudaFuncSetAttribute(sens_fwd_resident<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      sens_fwd_resident<32><<<grid, 512, smem, st>>>(a);
    }
    return cudaGetLastError();
  }
  const SensFwdGeom G = sens_fwd_geom(a.HP, a.D);
  const size_t smem = (size_t)G.DC * G.HPW * 16 + (size_t)G.DC * G.TR * 4;
  cudaError_t e = cudaFuncSetAttribute(sens_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long ntiles = (a.rows + G.TR - 1) / G.TR;
  const int per_sm = (G.NT <= 512 && smem <= 110 * 1024) ? 2 : 1;
  const long long grid = ntiles < (long long)num_sms * per_sm ? ntiles : (long long)num_sms * per_sm;
  sens_fwd_kernel<<<(int)grid, G.NT, smem, st>>>(a);
  return cudaGetLastError();
}

SensBwdPlan plan_sensory_bwd(long long rows, int D, int HP, int num_sms) {
  SensBwdPlan p{};
  p.qc = pick_qc(HP);
  p.nqc = HP / p.qc;
  p.dpc = 4096 / p.qc;
  p.ndc = (D + p.dpc - 1) / p.dpc;
  int ns = num_sms / (p.ndc * p.nqc);
  if (ns < 1) ns = 1;
  const long long max_split = (rows + kRT - 1) / kRT;
  if (ns > max_split) ns = (int)(max_split > 0 ? max_split : 1);
  p.nsplit = ns;
  p.part_floats = (size_t)ns * 4 * D * HP;
  p.dxpart_floats = p.nqc > 1 ? (size_t)p.nqc * rows * D : 0;
  return p;
}

cudaError_t launch_sensory_bwd(const SensBwdArgs& a, const SensBwdPlan& p, float* dxpart, bool tanh_space,
                               cudaStream_t st) {
  if (a.rows <= 0) return cudaSuccess;
  long long rps = (a.rows + p.nsplit - 1) / p.nsplit;
  rps = (rps + kRT - 1) / kRT * kRT;
  dim3 grid(p.ndc * p.nqc, p.nsplit);
  const size_t smem = 2 * ((size_t)2 * kRT * (p.qc + 4) * 4 + (size_t)kRT * p.dpc * 4);  // double-buffered
  cudaError_t e;
#define LTC_SB_CASE(QCV)                                                                                 \
  case QCV:                                                                                              \
    if (tanh_space) {                                                                                    \
      e = cudaFuncSetAttribute(sens_bwd_kernel<QCV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                               (int)smem);                                                              \
      if (e != cudaSuccess) return e;                                                                    \
      sens_bwd_kernel<QCV, true><<<grid, 256, smem, st>>>(a, p.nqc, rps, dxpart);                       \
    } else {                                                                                             \
      e = cudaFuncSetAttribute(sens_bwd_kernel<QCV, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,\
                               (int)smem);                                                              \
      if (e != cudaSuccess) return e;                                                                    \
      sens_bwd_kernel<QCV, false><<<grid, 256, smem, st>>>(a, p.nqc, rps, dxpart);                      \
    }                                                                                                    \
    break;
  switch (p.qc) {
    LTC_SB_CASE(32)
    LTC_SB_CASE(64)
    LTC_SB_CASE(128)
    LTC_SB_CASE(256)
    default:
      return cudaErrorInvalidValue;
  }
#undef LTC_SB_CASE
  return cudaGetLastError();
}

}  // namespace ltc
