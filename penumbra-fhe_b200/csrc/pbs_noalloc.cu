// pbs_noalloc.cu -- a bootstrap entry point that performs no device allocation.
//
// pnb_pbs_batch needs scratch (the keyswitched ciphertexts and the keyswitch digits).  Callers
// that hand it no workspace get that scratch from the stream-ordered allocator; callers that
// cannot allocate at all -- a host process whose GPU memory is already reserved by another
// framework's caching allocator, a serving loop that must not pay allocator latency or
// synchronisation on the request path, an FFI caller that has to keep its device footprint
// fixed after start-up -- use pnb_pbs_batch_noalloc instead.  Its scratch is the file-scope
// array below: 4 MiB, allocated once per GPU when the library's module is loaded there and held
// until the process exits.  With the default parameter set that holds 247 ciphertexts per call.
//
// Every call shares the array and finds the previous call's contents in it; the bootstrap
// writes every scratch word it reads, so nothing needs clearing.  Calls whose kernels overlap on
// the GPU (different streams, or different host threads) race on the array and must be
// serialised by the caller.
#include "pnb_internal.cuh"
#include "pnb_keys.h"

namespace pnb {

constexpr size_t NOALLOC_SCRATCH_BYTES = 4u << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_pbs_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_pbs_scratch on the current device.  Host code must not hand the symbol
// itself to a kernel: in host code it is only a stand-in for the device object.  The address is
// looked up on every call (the lookup allocates nothing), so a caller that resets the device or
// replaces its context never reaches a stale pointer.
static int noalloc_scratch(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_pbs_scratch);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(pbs scratch)");
  *out = p;
  return PNB_OK;
}

int pbs_batch_noalloc(const pnb_keys* K, const uint64_t* tv, const uint64_t* in, uint64_t* out,
                      int count, cudaStream_t st) {
  const size_t need = pbs_workspace_bytes(K, count);
  if (need > NOALLOC_SCRATCH_BYTES) {
    int max = count;
    while (max > 0 && pbs_workspace_bytes(K, max) > NOALLOC_SCRATCH_BYTES) --max;
    set_error("pbs_noalloc: %d ciphertexts need %zu bytes of scratch but the fixed scratch holds "
              "%zu bytes (at most %d ciphertexts with these keys); split the batch",
              count, need, NOALLOC_SCRATCH_BYTES, max);
    return PNB_ERR_INVALID;
  }
  if (!fft_tables_ready()) {
    set_error("pbs_noalloc: the FFT tables of this device are not built; create the key set "
              "with pnb_keygen or pnb_keys_import on this device first");
    return PNB_ERR_INVALID;
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return pbs_batch(K, tv, in, out, count, scratch, NOALLOC_SCRATCH_BYTES, st);
}

}  // namespace pnb
