// Sensory forward that skips structurally-zero sensory synapses (LTC_FLAG_SKIP_ZERO_SYNAPSES).
//
// A sensory synapse with sw = 0 (sensory_w_pos = softplus(w) * mask is zero where the
// mask is) adds nothing to sn = sum sw*serev*act or sd = sum sw*act, so the pass
// visits only the nonzero (d, q) pairs.  The forward values are those of the dense
// kernels up to summation order; no gradient changes (the backward does not read
// these tables).
//
// Tables (rebuilt on the device at every call, after the pack): for each column q the
// ascending list of its nonzero inputs d and their gate constants (the spack entries),
// and the column's weight sums.  One warp per column, a ballot per 32 inputs.
//
// Kernel: one warp per column, the lanes over rows (RPL rows each, one vector load of
// the transposed x tile per synapse), so a column's list is walked warp-uniformly and
// its constants are broadcast loads; no cross-lane reduction.  Outputs go through a
// shared-memory tile and leave as coalesced rows.
#include <cstdint>

#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace ltc {
namespace {

struct SensTablesView {
  int* cnt;       // [HP]     nonzero inputs of column q
  int* idx;       // [HP][D]  their indices d, ascending
  float4* cst;    // [HP][D]  spack[d][q] of each entry
  float2* cw;     // [HP]     (sum sw*serev, sum sw) over the column
};

inline size_t sens_layout(int D, int HP, size_t (&at)[4]) {
  const size_t sz[4] = {(size_t)HP * sizeof(int), (size_t)HP * D * sizeof(int), (size_t)HP * D * sizeof(float4),
                        (size_t)HP * sizeof(float2)};
  size_t o = 0;
  for (int i = 0; i < 4; ++i) {
    at[i] = o;
    o = (o + sz[i] + 255) & ~size_t(255);
  }
  return o;
}

inline SensTablesView sens_view(const void* base, int D, int HP) {
  char* b = static_cast<char*>(const_cast<void*>(base));
  size_t at[4];
  sens_layout(D, HP, at);
  SensTablesView v;
  v.cnt = reinterpret_cast<int*>(b + at[0]);
  v.idx = reinterpret_cast<int*>(b + at[1]);
  v.cst = reinterpret_cast<float4*>(b + at[2]);
  v.cw = reinterpret_cast<float2*>(b + at[3]);
  return v;
}

__global__ void __launch_bounds__(256) build_sens_kernel(SensTablesView tv, const float* __restrict__ sw,
                                                         const float4* __restrict__ spack, int D, int H, int HP) {
  const int q = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (q >= HP) return;
  int base = 0;
  float cwe = 0.f, cws = 0.f;
  for (int d0 = 0; d0 < D; d0 += 32) {
    const int d = d0 + lane;
    const bool on = q < H && d < D && sw[(long long)d * H + q] != 0.f;
    const unsigned m = __ballot_sync(0xffffffffu, on);
    if (on) {
      const int pos = base + __popc(m & ((1u << lane) - 1u));
      LTC_CHECK(pos < D, 301);
      const float4 k = spack[(long long)d * HP + q];
      tv.idx[(long long)q * D + pos] = d;
      tv.cst[(long long)q * D + pos] = k;
      cwe += k.w;
      cws += k.z;
    }
    base += __popc(m);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    cwe += __shfl_xor_sync(0xffffffffu, cwe, o);
    cws += __shfl_xor_sync(0xffffffffu, cws, o);
  }
  if (lane == 0) {
    tv.cnt[q] = base;
    tv.cw[q] = make_float2(cwe, cws);
  }
}

constexpr int kNT = 512, kQB = 32;  // threads; columns per output pass
constexpr int kLC = 128;            // list entries a warp stages in shared memory at a time

template <int RPL>
struct RowVec;
template <>
struct RowVec<2> {
  __device__ static void load(const float* p, float (&v)[2]) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x;
    v[1] = t.y;
  }
};
template <>
struct RowVec<4> {
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  }
};

__host__ __device__ constexpr size_t sens_sparse_smem(int D, int rpl, int nbuf) {
  return ((size_t)nbuf * D * 32 * rpl + (size_t)2 * 32 * rpl * (kQB + 1)) * sizeof(float) +
         (size_t)(kNT / 32) * kLC * (sizeof(float4) + sizeof(int));
}

// xs [nbuf][D][TR] (x tile transposed: row r of input d at d * TR + r), os [2][TR][kQB + 1],
// then per warp kLC list entries (constants, indices): a column's list is brought in
// with coalesced loads, kLC entries at a time, so the walk waits on no global load
template <int RPL>
__global__ void __launch_bounds__(kNT, 1) sens_fwd_sparse(SensFwdArgs a, SensTablesView tv, int nbuf) {
  constexpr int TR = 32 * RPL, LDO = kQB + 1;
  extern __shared__ __align__(16) float smem[];
  const int D = a.D, H = a.H;
  float* xs = smem;
  float* osn = xs + (size_t)nbuf * D * TR;
  float* osd = osn + TR * LDO;
  float4* lcs = reinterpret_cast<float4*>(osd + TR * LDO) + (threadIdx.x / 32) * kLC;
  int* lis = reinterpret_cast<int*>(reinterpret_cast<float4*>(osd + TR * LDO) + (kNT / 32) * kLC) +
             (threadIdx.x / 32) * kLC;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const long long ntiles = (a.rows + TR - 1) / TR;

  auto stage = [&](long long tile, int buf) {
    float* dst = xs + (size_t)buf * D * TR;
    const long long row0 = tile * TR;
    for (int i = tid; i < TR * D; i += kNT) {
      const int r = i % TR, d = i / TR;  // consecutive lanes -> consecutive rows: conflict-free stores
      const long long row = row0 + r;
      if (row < a.rows) cp_async4(dst + d * TR + r, a.x + row * D + d);
      else dst[d * TR + r] = 0.f;
    }
    cp_async_commit();
  };

  long long tile = blockIdx.x;
  if (tile < ntiles) stage(tile, 0);
  int buf = 0;
  for (; tile < ntiles; tile += gridDim.x) {
    cp_async_wait_all();
    __syncthreads();  // tile landed; with two buffers the other one is free again
    const bool more = tile + gridDim.x < ntiles;
    if (nbuf == 2 && more) stage(tile + gridDim.x, buf ^ 1);
    const float* xt = xs + (size_t)buf * D * TR + lane * RPL;
    const long long row0 = tile * TR;
    for (int q0 = 0; q0 < H; q0 += kQB) {
      for (int qq = warp; qq < kQB && q0 + qq < H; qq += kNT / 32) {
        const int q = q0 + qq;
        const int n = tv.cnt[q];
        const int* __restrict__ li = tv.idx + (long long)q * D;
        const float4* __restrict__ lc = tv.cst + (long long)q * D;
        float sn[RPL], sd[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) sn[i] = sd[i] = 0.f;
        auto visit = [&](int k, int xo) {  // xo: the entry's input d times TR
          const float4 w = lcs[k];
          float xv[RPL];
          RowVec<RPL>::load(xt + xo, xv);
#pragma unroll
          for (int i = 0; i < RPL; ++i) {
            const float th = tanh_approx(fmaf(w.x, xv[i], w.y));
            sn[i] = fmaf(w.w, th, sn[i]);
            sd[i] = fmaf(w.z, th, sd[i]);
          }
        };
        for (int base = 0; base < n; base += kLC) {
          const int m = min(kLC, n - base);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < kLC / 32; ++j) {
            const int k = j * 32 + lane;
            if (k < m) {
              lcs[k] = lc[base + k];
              int d = li[base + k];
              if (LTC_CHECKED_SKIP(d >= 0 && d < D, 302)) d = 0;
              lis[k] = d * TR;
            }
          }
          __syncwarp();
          int k = 0;
          for (; k + 3 < m; k += 4) {
            const int4 xo = *reinterpret_cast<const int4*>(lis + k);  // four offsets, one load
            visit(k, xo.x);
            visit(k + 1, xo.y);
            visit(k + 2, xo.z);
            visit(k + 3, xo.w);
          }
          for (; k < m; ++k) visit(k, lis[k]);
        }
        const float2 cw = tv.cw[q];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {  // act = 1/2 + tanh/2: the constant half is the column sum
          osn[(lane * RPL + i) * LDO + qq] = 0.5f * (cw.x + sn[i]);
          osd[(lane * RPL + i) * LDO + qq] = 0.5f * (cw.y + sd[i]);
        }
      }
      __syncthreads();
      const int qn = min(kQB, H - q0);
      for (int i = tid; i < TR * kQB; i += kNT) {
        const int r = i / kQB, qq = i % kQB;
        const long long row = row0 + r;
        if (qq < qn && row < a.rows) {
          a.sn[row * H + q0 + qq] = osn[r * LDO + qq];
          a.sd[row * H + q0 + qq] = osd[r * LDO + qq];
        }
      }
      __syncthreads();
    }
    if (nbuf == 2) {
      buf ^= 1;
    } else if (more) {
      stage(tile + gridDim.x, 0);
    }
  }
  cp_async_wait_all();
}

}  // namespace

size_t sens_tables_bytes(int D, int HP) {
  size_t at[4];
  return sens_layout(D, HP, at);
}

cudaError_t launch_build_sens(const PackArgs& pa, void* tables, cudaStream_t st) {
  const SensTablesView tv = sens_view(tables, pa.D, pa.HP);
  const int warps_per_block = 8;
  build_sens_kernel<<<(pa.HP + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, st>>>(
      tv, pa.sw, pa.spack, pa.D, pa.H, pa.HP);
  return cudaGetLastError();
}

bool sens_sparse_fits(int D) { return sens_sparse_smem(D, 2, 1) <= 227 * 1024; }

cudaError_t launch_sensory_fwd_sparse(const SensFwdArgs& a, const void* tables, int num_sms, cudaStream_t st) {
  if (a.rows <= 0) return cudaSuccess;
  const SensTablesView tv = sens_view(tables, a.D, a.HP);
  const size_t cap = 227 * 1024;
  // widest row vectors first, double-buffered when it fits
  int rpl = 0, nbuf = 0;
  const int cand[4][2] = {{4, 2}, {4, 1}, {2, 2}, {2, 1}};
  for (auto& c : cand)
    if (sens_sparse_smem(a.D, c[0], c[1]) <= cap) {
      rpl = c[0];
      nbuf = c[1];
      break;
    }
  if (!rpl) return cudaErrorInvalidValue;
  const size_t smem = sens_sparse_smem(a.D, rpl, nbuf);
  const long long ntiles = (a.rows + 32 * rpl - 1) / (32 * rpl);
  const int grid = (int)(ntiles < num_sms ? ntiles : num_sms);
  cudaError_t e;
  if (rpl == 4) {
    e = cudaFuncSetAttribute(sens_fwd_sparse<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sens_fwd_sparse<4><<<grid, kNT, smem, st>>>(a, tv, nbuf);
  } else {
    e = cudaFuncSetAttribute(sens_fwd_sparse<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sens_fwd_sparse<2><<<grid, kNT, smem, st>>>(a, tv, nbuf);
  }
  return cudaGetLastError();
}

}  // namespace ltc
