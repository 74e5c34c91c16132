// scmp_sc_matmul_noalloc: the sc_matmul pipeline with library-owned scratch.
//
// scmp_sc_matmul takes its scratch (quantised operands, row statistics and
// scales) from a workspace the caller allocates. Some callers cannot do that:
// a host program that reaches this library through a plain C FFI and has no
// device allocator of its own, or a serving process that reserved all of its
// device memory up front and must not call cudaMalloc later (the call can
// also synchronise the whole device). For them this entry point runs the same
// kernels on a fixed scratch array that lives in the library's device image.
//
// The array below is kNoAllocScratchBytes (16 MiB) on every GPU that loads
// the library, held until the process exits. Host code cannot use its name as
// a device address, so the first call on each device, with that device
// current, looks the address up with cudaGetSymbolAddress and caches it; make
// that first call before any stream capture. Calls whose workspace would
// exceed the array are rejected. All calls share the array and it keeps the
// last call's contents; every value the pipeline reads from it is written
// earlier in the same call, so nothing needs clearing, but two calls on the
// same device that overlap on the GPU (for example on two streams with no
// ordering between them) race on it. Each device has its own copy.
#include <mutex>
#include <string>

namespace scmp {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[128];  // per device ordinal, filled on first use

static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "sc_matmul_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 128) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "sc_matmul_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SCMP_OK;
}

}  // namespace scmp

extern "C" int scmp_sc_matmul_noalloc(const scmp_matmul_desc* desc, void* stream) {
  using namespace scmp;
  size_t need = 0;
  int s = scmp_sc_matmul_workspace_size(desc, &need);
  if (s) return s;
  if (desc->flags & SCMP_FLAG_B_READY)  // the shared array keeps no weight between calls
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_noalloc: SCMP_FLAG_B_READY needs a caller-owned workspace");
  scmp_matmul_desc whole;
  if (need > kNoAllocScratchBytes && !(desc->flags & SCMP_FLAG_NO_SPLIT)) {
    // without the split last wave's part accumulators the call may still fit
    whole = *desc;
    whole.flags |= SCMP_FLAG_NO_SPLIT;
    desc = &whole;
    s = scmp_sc_matmul_workspace_size(desc, &need);
    if (s) return s;
  }
  if (need > kNoAllocScratchBytes)
    return fail(SCMP_ERR_INVALID_ARG,
                "sc_matmul_noalloc: this call needs " + std::to_string(need) +
                    " bytes of scratch, more than the fixed 16 MiB array; use scmp_sc_matmul "
                    "with a caller-provided workspace");
  void* scratch = nullptr;
  s = noalloc_scratch(&scratch);
  if (s) return s;
  return scmp_sc_matmul(desc, scratch, kNoAllocScratchBytes, stream);
}
