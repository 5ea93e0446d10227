// Parameter packing (run once per call, in front of the solver kernels) and the
// deterministic gradient reduction + transforms that close the backward pass.
#include "ltc_common.cuh"
#include "ltc_internal.h"

namespace ltc {

// Gate packs (sh, nh, w, w*erev) with zero padding up to HP; see ltc_common.cuh.
__global__ void pack_kernel(PackArgs a) {
  // a null w_pos (sigma) skips the recurrent (sensory) packs: step-level calls
  const long long nrec = a.w_pos ? (long long)a.HP * a.HP : 0;
  const long long nsen = a.ssig ? (long long)a.D * a.HP : 0;
  const long long total = nrec + nsen + (a.cm ? a.HP : 0);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < nrec) {
      const int p = (int)(i / a.HP), q = (int)(i % a.HP);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p < a.H && q < a.H) {
        const long long j = (long long)p * a.H + q;
        const float sg = a.sigma[j];
        v.x = 0.5f * sg;
        v.y = -0.5f * sg * a.mu[j];
        v.z = a.w_pos[j];
        v.w = a.w_erev[j];
      }
      a.pack[i] = v;
      if (a.packT) {
        if (a.packT_qc > 0) {
          const int qc = a.packT_qc, c = q % qc;
          a.packT[(long long)p * a.HP + (q - c) + (c % 8) * (qc / 8) + c / 8] = v;
        } else {
          a.packT[(long long)q * a.HP + p] = v;
        }
      }
    } else if (i < nrec + nsen) {
      const long long k = i - nrec;
      const int d = (int)(k / a.HP), q = (int)(k % a.HP);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q < a.H) {
        const long long j = (long long)d * a.H + q;
        const float sg = a.ssig[j];
        v.x = 0.5f * sg;
        v.y = -0.5f * sg * a.smu[j];
        v.z = a.sw[j];
        v.w = a.sw[j] * a.serev[j];
      }
      a.spack[k] = v;
    } else {
      const int q = (int)(i - nrec - nsen);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q < a.H) {
        v.x = a.cm[q];
        v.y = a.gl[q];
        v.z = a.vl[q];
        v.w = a.gl[q] * a.vl[q];
      }
      a.nrn[q] = v;
    }
  }
}

cudaError_t launch_pack(const PackArgs& a, cudaStream_t st) {
  const long long total = (a.w_pos ? (long long)a.HP * a.HP : 0) + (a.ssig ? (long long)a.D * a.HP : 0) +
                          (a.cm ? a.HP : 0);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (int)((total + threads - 1) / threads < 4096 ? (total + threads - 1) / threads : 4096);
  pack_kernel<<<blocks, threads, 0, st>>>(a);
  return cudaGetLastError();
}

// Fixed-order sums over the per-CTA partial slabs, then the closed-form
// transforms from the accumulated sums to the solver-input gradients:
//   recurrent  g_w_erev = S0, g_w_pos = S1, g_mu = -sigma*S2, g_sigma = S3 - mu*S2
//   sensory    g_serev = sw*A_n, g_sw = serev*A_n + A_d, g_smu = -ssig*DZ, g_ssig = DZX - smu*DZ
// where S2/DZ = sum of dL/dz and S3/DZX = sum of dL/dz * (presynaptic value).
__global__ void finish_kernel(FinishArgs a) {
  // a null rec_part (sens_part) skips the recurrent (sensory) outputs: step-level calls
  const long long nrec = a.rec_part ? (long long)a.H * a.H : 0;
  const long long nneu = a.rec_part ? a.H : 0;
  const long long nsen = a.sens_part ? (long long)a.D * a.H : 0;
  const long long ndx = (a.nqc > 1) ? a.rows * a.D : 0;
  const long long total = nrec + nneu + nsen + ndx;
  const long long hp2 = (long long)a.HP * a.HP;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < nrec) {
      const int p = (int)(i / a.H), q = (int)(i % a.H);
      if (a.skip_w_pos && a.skip_w_pos[i] == 0.f && a.skip_w_erev[i] == 0.f) {
        a.g_w_erev[i] = a.g_w_pos[i] = a.g_mu[i] = a.g_sigma[i] = 0.f;
        continue;
      }
      const long long idx = a.rec_transposed ? (long long)q * a.HP + p : (long long)p * a.HP + q;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      for (int c = 0; c < a.rslots; ++c) {
        const float* base = a.rec_part + (long long)c * 4 * hp2 + idx;
        s0 += base[0];
        s1 += base[hp2];
        s2 += base[2 * hp2];
        s3 += base[3 * hp2];
      }
      if (a.rec_tanh_space) {
        // sum a*act = sum a/2 + 2 * sum a'*tanh  with a' = -a/4, tanh = tanh(-z/2)
        float san = 0.f, sad = 0.f;
        for (int c = 0; c < a.rslots; ++c) {
          san += a.rec_partn[((long long)c * 5 + 3) * a.HP + q];
          sad += a.rec_partn[((long long)c * 5 + 4) * a.HP + q];
        }
        s0 = fmaf(0.5f, san, 2.0f * s0);
        s1 = fmaf(0.5f, sad, 2.0f * s1);
      }
      a.g_w_erev[i] = s0;
      a.g_w_pos[i] = s1;
      a.g_mu[i] = -a.sigma[i] * s2;
      a.g_sigma[i] = s3 - a.mu[i] * s2;
    } else if (i < nrec + nneu) {
      const int q = (int)(i - nrec);
      const int kn = a.rec_tanh_space ? 5 : 3;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f;
      for (int c = 0; c < a.rslots; ++c) {
        const float* base = a.rec_partn + (long long)c * kn * a.HP + q;
        s0 += base[0];
        s1 += base[a.HP];
        s2 += base[2 * a.HP];
      }
      a.g_cm[q] = s0;
      a.g_gl[q] = s1;
      a.g_vl[q] = s2;
    } else if (i < nrec + nneu + nsen) {
      const long long k = i - nrec - nneu;
      const int d = (int)(k / a.H), q = (int)(k % a.H);
      if (a.skip_sw && a.skip_sw[k] == 0.f) {
        a.g_serev[k] = a.g_sw[k] = a.g_smu[k] = a.g_ssig[k] = 0.f;
        continue;
      }
      const long long idx = (long long)d * a.HP + q;
      const long long slab = (long long)a.D * a.HP;
      float an = 0.f, ad = 0.f, dz = 0.f, dzx = 0.f;
      for (int c = 0; c < a.nsplit; ++c) {
        const float* base = a.sens_part + (long long)c * 4 * slab + idx;
        an += base[0];
        ad += base[slab];
        dz += base[2 * slab];
        dzx += base[3 * slab];
      }
      if (a.rec_tanh_space) {
        // sum g*act = sum g/2 + 2 * sum a'*tanh; sum over rows of g_sn = sum of a_n
        float san = 0.f, sad = 0.f;
        for (int c = 0; c < a.rslots; ++c) {
          san += a.rec_partn[((long long)c * 5 + 3) * a.HP + q];
          sad += a.rec_partn[((long long)c * 5 + 4) * a.HP + q];
        }
        an = fmaf(0.5f, san, 2.0f * an);
        ad = fmaf(0.5f, sad, 2.0f * ad);
      }
      a.g_serev[k] = a.sw[k] * an;
      a.g_sw[k] = a.serev[k] * an + ad;
      a.g_smu[k] = -a.ssig[k] * dz;
      a.g_ssig[k] = dzx - a.smu[k] * dz;
    } else {
      const long long k = i - nrec - nneu - nsen;
      float s = 0.f;
      for (int c = 0; c < a.nqc; ++c) s += a.dxpart[(long long)c * ndx + k];
      a.g_x[k] = s;
    }
  }
}

cudaError_t launch_finish(const FinishArgs& a, int num_sms, cudaStream_t st) {
  const long long total = (a.rec_part ? (long long)a.H * a.H + a.H : 0) + (a.sens_part ? (long long)a.D * a.H : 0) +
                          ((a.nqc > 1) ? a.rows * a.D : 0);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
  if (blocks < 1) blocks = 1;
  finish_kernel<<<(int)blocks, threads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace ltc
