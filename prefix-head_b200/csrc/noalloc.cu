// gem_head_full_noalloc: the batched full head (gem_head_full_dev) for callers that cannot allocate
// device memory at call time.
//
// Some callers cannot call cudaMalloc when they score: a process whose device memory is owned by
// another allocator (a framework's caching pool, an inference server that pre-plans every byte), a
// real-time loop that must not block in the driver's allocator, or code that runs while another
// component is capturing work on the stream. gem_head_full_dev allocates its quantized-activation and
// per-CTA partial buffers per call; this variant keeps them in one static device array instead.
//
// The array is a file-scope __device__ object of kScratchBytes (1 MiB): every GPU that loads this
// library holds it until the process exits. Host code cannot use the array's name as a device address
// (on the host it names a host-side stand-in), so the first call on each device, with that device
// current, resolves the address with cudaGetSymbolAddress and caches it. Make that first call before
// any stream capture. Every call on a device shares the array and it keeps the last call's contents:
// calls whose work overlaps on the GPU (two streams, two threads, two models on one device) race on it.
// Each launch overwrites every scratch element it later reads, so nothing needs clearing between calls.
#include <mutex>
#include <string>

#include "../../include/gem.h"
#include "internal.hpp"
#include "kernels.cuh"

namespace {

constexpr size_t kScratchBytes = 1u << 20;
static __device__ __align__(256) unsigned char g_head_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

size_t align16(size_t x) { return (x + 15) / 16 * 16; }

// Device address of g_head_scratch on `device` (which must be current).
int scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) {
    gem::set_last_error("device index out of range for the no-allocation scratch");
    return GEM_E_ARG;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_head_scratch);
    if (e != cudaSuccess || !p) {
      gem::set_last_error(std::string("cudaGetSymbolAddress(no-allocation scratch): ") + cudaGetErrorString(e));
      return GEM_E_CUDA;
    }
    g_scratch_addr[device] = p;
  }
  *out = (unsigned char*)g_scratch_addr[device];
  return GEM_OK;
}

}  // namespace

extern "C" int gem_head_full_noalloc(gem_model* m, const float* h_dev, const uint32_t* targets_dev, int batch,
                                     float* logprob_dev, uint32_t* argmax_dev) {
  gem::ModelHeadView v;
  if (!m || !h_dev || !targets_dev || !logprob_dev || batch <= 0 || !gem::model_head_view(m, &v)) {
    gem::set_last_error("null argument or batch <= 0");
    return GEM_E_ARG;
  }
  const int parts = gem::head_full_parts(v.sms);
  const size_t q_bytes = align16((size_t)batch * v.d);
  const size_t s_bytes = align16((size_t)batch * (v.d / 32) * sizeof(float));
  const size_t part_bytes = (size_t)batch * parts * 4 * sizeof(float);
  const size_t t_bytes = align16((size_t)batch * sizeof(float));
  const size_t need = q_bytes + s_bytes + part_bytes + t_bytes;
  if (need > kScratchBytes) {
    const size_t per_item = v.d + (v.d / 32) * sizeof(float) + (size_t)parts * 16 + sizeof(float);
    gem::set_last_error("batch " + std::to_string(batch) + " needs " + std::to_string(need) +
                        " bytes of scratch; the no-allocation head has " + std::to_string(kScratchBytes) +
                        " (about " + std::to_string(kScratchBytes / per_item) + " hidden states for this model)");
    return GEM_E_ARG;
  }
  cudaError_t e = cudaSetDevice(v.device);
  if (e != cudaSuccess) {
    gem::set_last_error(std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    return GEM_E_CUDA;
  }
  unsigned char* base = nullptr;
  int rc = scratch_address(v.device, &base);
  if (rc != GEM_OK) return rc;
  int8_t* q = (int8_t*)base;
  float* s = (float*)(base + q_bytes);
  float* part = (float*)(base + q_bytes + s_bytes);
  float* tlogit = (float*)(base + q_bytes + s_bytes + part_bytes);

  gem::launch_quantize(h_dev, batch * v.d, q, s, v.st);
  gem::HeadArgs H{};
  H.w = v.w;
  H.row_of = v.row_of, H.row_tok = v.row_tok;
  H.aq = q, H.as = s, H.h = h_dev;
  H.targets = targets_dev;
  H.part = part;
  H.tlogit = tlogit;
  H.lp_out = logprob_dev;
  H.am_out = argmax_dev;
  H.err = v.err;
  if (v.exact) gem::launch_head_full_exact(H, batch, v.sms, v.st);
  else gem::launch_head_full(H, batch, v.sms, v.st);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    gem::set_last_error(std::string("kernel launch: ") + cudaGetErrorString(e));
    return GEM_E_CUDA;
  }
  return GEM_OK;
}
