// ltc_forward_noalloc: the forward solve with no allocation of any kind.
//
// Who needs this: callers that are not allowed to allocate GPU memory at the
// point where they run the solver.  Examples are hosts that hand the library
// only their own tensors and keep every allocation under their control (a
// plugin inside a serving runtime with a fixed memory budget, or a framework
// whose allocator owns the device), and latency-critical loops in which a
// cudaMalloc would synchronise the device.  ltc_forward() needs a workspace
// from the caller; this variant needs none: its scratch (gate packs and the
// sensory sums) lives in one file-scope __device__ array of
// LTC_NOALLOC_SCRATCH_BYTES that every GPU which loads the library holds
// until the process exits.  It saves no state for a backward pass.
//
// Rules of use:
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (the host-side name of a __device__ array is only a
//    stand-in, never a device pointer).  Make that first call before any
//    stream capture.
//  * All calls on a device share the one array, which keeps whatever the last
//    call left in it.  Every byte a call reads is written earlier in the same
//    call (pack -> sensory sums -> solve), so nothing needs clearing, but two
//    calls that overlap on the GPU (different streams, or host threads racing)
//    race on the array: serialise them.
//  * Problems whose scratch exceeds LTC_NOALLOC_SCRATCH_BYTES are rejected
//    with an error (see ltc_last_error) before any GPU work is queued.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/ltc_sm100.h"
#include "ltc_internal.h"

using namespace ltc;

static __device__ __align__(256) unsigned char g_noalloc_scratch[LTC_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

int noalloc_fail(const char* msg) {
  set_last_error(msg);
  return 1;
}

// Device address of g_noalloc_scratch for the current device (looked up once per device).
int scratch_address(int dev, unsigned char** out) {
  static std::mutex mu;
  static unsigned char* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char buf[256];
      snprintf(buf, sizeof(buf), "ltc_forward_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return noalloc_fail(buf);
    }
    addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = addr[dev];
  return 0;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

extern "C" int ltc_forward_noalloc(const LtcDims* dims, const LtcParams* params, const float* x, const float* h0,
                                   float* outputs, float* h_final, ltc_stream_t stream) {
  if (!dims || !params || !x || !outputs || !h_final) return noalloc_fail("ltc_forward_noalloc: NULL argument");
  const LtcParams& p = *params;
  if (!p.w_pos || !p.w_erev || !p.mu || !p.sigma || !p.sensory_mu || !p.sensory_sigma || !p.sensory_erev ||
      !p.sensory_w_pos || !p.cm_t || !p.gleak_pos || !p.vleak)
    return noalloc_fail("ltc_forward_noalloc: a parameter pointer is NULL");
  const int B = dims->B, T = dims->T, D = dims->D, H = dims->H, U = dims->ode_unfolds;
  if (B < 1 || T < 1 || D < 1 || H < 1 || U < 1 || H > 512)
    return noalloc_fail("ltc_forward_noalloc: invalid dims (need B,T,D,H,ode_unfolds >= 1 and H <= 512)");
  int dev = 0, sms = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return noalloc_fail("ltc_forward_noalloc: no current CUDA device");
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
    return noalloc_fail("ltc_forward_noalloc: requires an sm_100 (B200-class) GPU");

  const RecPlan rp = plan_recurrent(B, H, sms, dims->flags & LTC_FLAG_FORCE_WIDE);
  const int HP = rp.HP;
  const long long rows = (long long)B * T;
  // scratch layout: pack [HP*HP] float4 | spack [D*HP] float4 | nrn [HP] float4 | sn [rows*H] | sd [rows*H]
  //                 | recurrent-kernel scratch (the streamed path for H > 128)
  const size_t o_pack = 0;
  const size_t o_spack = align256(o_pack + (size_t)HP * HP * sizeof(float4));
  const size_t o_nrn = align256(o_spack + (size_t)D * HP * sizeof(float4));
  const size_t o_sn = align256(o_nrn + (size_t)HP * sizeof(float4));
  const size_t o_sd = align256(o_sn + (size_t)rows * H * sizeof(float));
  const size_t o_scr = align256(o_sd + (size_t)rows * H * sizeof(float));
  const size_t need = o_scr + rp.scratch_fwd * sizeof(float);
  if (need > (size_t)LTC_NOALLOC_SCRATCH_BYTES) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "ltc_forward_noalloc: problem needs %zu bytes of scratch, above the fixed %u-byte limit "
             "(use ltc_forward with a caller workspace)",
             need, (unsigned)LTC_NOALLOC_SCRATCH_BYTES);
    return noalloc_fail(buf);
  }
  unsigned char* base = nullptr;
  if (scratch_address(dev, &base)) return 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  PackArgs pa{};
  pa.w_pos = p.w_pos; pa.w_erev = p.w_erev; pa.mu = p.mu; pa.sigma = p.sigma;
  pa.smu = p.sensory_mu; pa.ssig = p.sensory_sigma; pa.serev = p.sensory_erev; pa.sw = p.sensory_w_pos;
  pa.cm = p.cm_t; pa.gl = p.gleak_pos; pa.vl = p.vleak;
  pa.pack = reinterpret_cast<float4*>(base + o_pack);
  pa.packT = nullptr;
  pa.spack = reinterpret_cast<float4*>(base + o_spack);
  pa.nrn = reinterpret_cast<float4*>(base + o_nrn);
  pa.D = D; pa.H = H; pa.HP = HP;
  cudaError_t e = launch_pack(pa, st);
  if (e == cudaSuccess) {
    SensFwdArgs sa{};
    sa.spack = pa.spack; sa.x = x;
    sa.sn = reinterpret_cast<float*>(base + o_sn);
    sa.sd = reinterpret_cast<float*>(base + o_sd);
    sa.rows = rows; sa.D = D; sa.H = H; sa.HP = HP;
    e = launch_sensory_fwd(sa, sms, st);
    if (e == cudaSuccess) {
      RecFwdArgs ra{};
      ra.pack = pa.pack; ra.nrn = pa.nrn; ra.sn = sa.sn; ra.sd = sa.sd; ra.h0 = h0;
      ra.out = outputs; ra.hT = h_final; ra.V = nullptr; ra.R = nullptr;
      ra.B = B; ra.T = T; ra.H = H; ra.U = U; ra.HP = HP; ra.ns = rp.ns_fwd; ra.eps = dims->epsilon;
      ra.scratch = rp.scratch_fwd ? reinterpret_cast<float*>(base + o_scr) : nullptr;
      e = launch_recurrent_fwd(ra, rp, st);
    }
  }
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "ltc_forward_noalloc: launch failed: %s", cudaGetErrorString(e));
    return noalloc_fail(buf);
  }
  set_last_error("");
  return 0;
}
