// capi.cu -- the extern "C" entry points declared in include/penumbra_b200.h.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>

#include "pnb_internal.cuh"
#include "pnb_keys.h"

namespace pnb {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return e == cudaErrorMemoryAllocation ? PNB_ERR_OOM : PNB_ERR_CUDA;
}

// Switch to the key set's device for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  int rc = PNB_OK;
  explicit DeviceGuard(int dev) {
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) { rc = cuda_status(e, "cudaGetDevice"); return; }
    if (prev != dev) {
      e = cudaSetDevice(dev);
      if (e != cudaSuccess) rc = cuda_status(e, "cudaSetDevice");
    }
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

static int validate_params(const pnb_params* p) {
  if (!p) { set_error("params is NULL"); return PNB_ERR_INVALID; }
  auto pow2 = [](int v) { return v > 0 && (v & (v - 1)) == 0; };
  if (p->n <= 0 || p->k <= 0 || !pow2(p->N) || p->N < 64) {
    set_error("params: need n > 0, k > 0, N a power of two >= 64 (got n=%d k=%d N=%d)", p->n,
              p->k, p->N);
    return PNB_ERR_INVALID;
  }
  if (p->pbs_base_log <= 0 || p->pbs_level <= 0 || p->pbs_base_log * p->pbs_level >= 64 ||
      p->ks_base_log <= 0 || p->ks_level <= 0 || p->ks_base_log * p->ks_level >= 64) {
    set_error("params: gadget base_log * level must be in [1, 63]");
    return PNB_ERR_INVALID;
  }
  if (p->msg_bits < 0 || p->carry_bits < 0 || p->msg_bits + p->carry_bits < 1 ||
      p->msg_bits + p->carry_bits > 16) {
    set_error("params: msg_bits + carry_bits must be in [1, 16]");
    return PNB_ERR_INVALID;
  }
  if (!(p->lwe_std >= 0.0) || !(p->glwe_std >= 0.0) || p->lwe_std >= 0.5 ||
      p->glwe_std >= 0.5) {
    set_error("params: noise std must be in [0, 0.5)");
    return PNB_ERR_INVALID;
  }
  return PNB_OK;
}

static int check_keys(const pnb_keys* K) {
  if (!K) { set_error("keys is NULL"); return PNB_ERR_INVALID; }
  return PNB_OK;
}

// Client-side operations need the secret keys, which an imported evaluation-key set may lack.
static int check_secret(const pnb_keys* K, bool small) {
  if (small ? !K->lwe_sk : !K->glwe_sk) {
    set_error("this key set holds no %s secret key (evaluation keys imported without it)",
              small ? "small" : "big");
    return PNB_ERR_INVALID;
  }
  return PNB_OK;
}

// Device buffers of a key set for `p` (secret keys only when asked for).
static int alloc_keys(pnb_keys* K, const pnb_params& p, bool with_secrets) {
  const size_t rows = (size_t)(p.k + 1) * p.pbs_level;
  K->bsk_words = (size_t)p.n * rows * (p.k + 1) * p.N;
  K->fbsk_elems = K->bsk_words / 2;
  K->ksk_row = (p.n + 2) & ~1;
  K->ksk_words = (size_t)p.k * p.N * p.ks_level * K->ksk_row;
  cudaError_t e = cudaSuccess;
  if ((with_secrets && ((e = cudaMalloc(&K->lwe_sk, sizeof(uint64_t) * p.n)) != cudaSuccess ||
                        (e = cudaMalloc(&K->glwe_sk, sizeof(uint64_t) * p.k * p.N)) !=
                            cudaSuccess)) ||
      (e = cudaMalloc(&K->bsk, sizeof(uint64_t) * K->bsk_words)) != cudaSuccess ||
      (e = cudaMalloc(&K->fbsk, sizeof(double2) * K->fbsk_elems)) != cudaSuccess ||
      (e = cudaMalloc(&K->ksk, sizeof(uint64_t) * K->ksk_words)) != cudaSuccess)
    return cuda_status(e, "cudaMalloc(keys)");
  return PNB_OK;
}

}  // namespace pnb

using namespace pnb;

extern "C" {

int pnb_version(void) { return 100; }

const char* pnb_last_error(void) { return g_err; }

int pnb_params_default(pnb_params* out) {
  if (!out) { set_error("out is NULL"); return PNB_ERR_INVALID; }
  memset(out, 0, sizeof(*out));
  out->n = 834;
  out->k = 1;
  out->N = 2048;
  out->pbs_base_log = 23;
  out->pbs_level = 1;
  out->ks_base_log = 3;
  out->ks_level = 5;
  out->msg_bits = 2;
  out->carry_bits = 2;
  out->lwe_std = 3.5539902359442825e-06;
  out->glwe_std = 2.845267479601915e-15;
  return PNB_OK;
}

int pnb_params_n8192(pnb_params* out) {
  if (!out) { set_error("out is NULL"); return PNB_ERR_INVALID; }
  memset(out, 0, sizeof(*out));
  out->n = 1024;
  out->k = 1;
  out->N = 8192;
  out->pbs_base_log = 23;
  out->pbs_level = 1;
  out->ks_base_log = 4;
  out->ks_level = 5;
  out->msg_bits = 3;
  out->carry_bits = 3;
  out->lwe_std = 2.9802322387695312e-08;  // 2^-25
  out->glwe_std = 2.168404344971009e-19;  // 2^-62
  return PNB_OK;
}

int pnb_keygen(int device, const pnb_params* params, uint64_t seed, pnb_keys** out) {
  if (!out) { set_error("out is NULL"); return PNB_ERR_INVALID; }
  *out = nullptr;
  int rc = validate_params(params);
  if (rc) return rc;
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  pnb_keys* K = new (std::nothrow) pnb_keys();
  if (!K) { set_error("host allocation failed"); return PNB_ERR_OOM; }
  K->device = device;
  K->p = *params;
  K->seed = seed;
  const pnb_params& p = *params;
  rc = alloc_keys(K, p, true);
  if (rc) {
    pnb_keys_free(K);
    return rc;
  }
  cudaError_t e;
  cudaStream_t st = 0;
  rc = keygen_device(K, st);
  if (rc == PNB_OK && p.N == 2048) {
    rc = bsk_to_fourier(K->bsk, K->fbsk, (int)(K->bsk_words / p.N), st);
  } else if (rc == PNB_OK && p.N == 8192) {
    rc = bsk_to_fourier_8k(K->bsk, K->fbsk, (int)(K->bsk_words / p.N), st);
  }
  if (rc == PNB_OK) {
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = cuda_status(e, "keygen synchronize");
  }
  if (rc) { pnb_keys_free(K); return rc; }
  *out = K;
  return PNB_OK;
}

int pnb_keys_import(int device, const pnb_params* params, const uint64_t* lwe_sk,
                    const uint64_t* glwe_sk, const uint64_t* bsk, const uint64_t* ksk,
                    pnb_keys** out) {
  if (!out) { set_error("out is NULL"); return PNB_ERR_INVALID; }
  *out = nullptr;
  if (!bsk || !ksk) {
    set_error("pnb_keys_import: the bootstrapping and keyswitching keys are required");
    return PNB_ERR_INVALID;
  }
  if (!lwe_sk != !glwe_sk) {
    set_error("pnb_keys_import: give both secret keys or neither");
    return PNB_ERR_INVALID;
  }
  int rc = validate_params(params);
  if (rc) return rc;
  if (params->N != 2048 && params->N != 8192) {
    set_error("pnb_keys_import: the Fourier conversion is compiled for N = 2048 and 8192 (got %d)",
              params->N);
    return PNB_ERR_UNSUPPORTED;
  }
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  pnb_keys* K = new (std::nothrow) pnb_keys();
  if (!K) { set_error("host allocation failed"); return PNB_ERR_OOM; }
  K->device = device;
  K->p = *params;
  K->seed = 0;
  const pnb_params& p = *params;
  rc = alloc_keys(K, p, lwe_sk != nullptr);
  cudaError_t e = cudaSuccess;
  if (rc == PNB_OK && lwe_sk) {
    if ((e = cudaMemcpy(K->lwe_sk, lwe_sk, 8 * (size_t)p.n, cudaMemcpyHostToDevice)) !=
            cudaSuccess ||
        (e = cudaMemcpy(K->glwe_sk, glwe_sk, 8 * (size_t)p.k * p.N, cudaMemcpyHostToDevice)) !=
            cudaSuccess)
      rc = cuda_status(e, "pnb_keys_import(secret keys)");
  }
  if (rc == PNB_OK &&
      (e = cudaMemcpy(K->bsk, bsk, 8 * K->bsk_words, cudaMemcpyHostToDevice)) != cudaSuccess)
    rc = cuda_status(e, "pnb_keys_import(bootstrapping key)");
  if (rc == PNB_OK) {
    // rows of n+1 words on the host, padded to ksk_row words on the device (pad words zero)
    const size_t rows = (size_t)p.k * p.N * p.ks_level;
    if ((e = cudaMemset(K->ksk, 0, 8 * K->ksk_words)) != cudaSuccess ||
        (e = cudaMemcpy2D(K->ksk, 8 * (size_t)K->ksk_row, ksk, 8 * (size_t)(p.n + 1),
                          8 * (size_t)(p.n + 1), rows, cudaMemcpyHostToDevice)) != cudaSuccess)
      rc = cuda_status(e, "pnb_keys_import(keyswitching key)");
  }
  if (rc == PNB_OK)
    rc = p.N == 8192 ? bsk_to_fourier_8k(K->bsk, K->fbsk, (int)(K->bsk_words / p.N), 0)
                     : bsk_to_fourier(K->bsk, K->fbsk, (int)(K->bsk_words / p.N), 0);
  if (rc == PNB_OK && (e = cudaStreamSynchronize(0)) != cudaSuccess)
    rc = cuda_status(e, "pnb_keys_import synchronize");
  if (rc) {
    pnb_keys_free(K);
    return rc;
  }
  *out = K;
  return PNB_OK;
}

int pnb_keys_free(pnb_keys* K) {
  if (!K) return PNB_OK;
  DeviceGuard g(K->device);
  cudaFree(K->lwe_sk);
  cudaFree(K->glwe_sk);
  cudaFree(K->bsk);
  cudaFree(K->fbsk);
  cudaFree(K->ksk);
  delete K;
  return PNB_OK;
}

int pnb_keys_info(const pnb_keys* K, pnb_params* params_out, int* device_out,
                  size_t* fourier_bsk_bytes, size_t* ksk_bytes) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (params_out) *params_out = K->p;
  if (device_out) *device_out = K->device;
  if (fourier_bsk_bytes) *fourier_bsk_bytes = K->fbsk_elems * sizeof(double2);
  if (ksk_bytes) *ksk_bytes = K->ksk_words * sizeof(uint64_t);
  return PNB_OK;
}

int pnb_keys_export(const pnb_keys* K, uint64_t* lwe_sk, uint64_t* glwe_sk, uint64_t* bsk,
                    uint64_t* ksk) {
  int rc = check_keys(K);
  if (rc) return rc;
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  const pnb_params& p = K->p;
  if ((lwe_sk || glwe_sk) && (rc = check_secret(K, false))) return rc;
  if (lwe_sk) PNB_CUDA(cudaMemcpy(lwe_sk, K->lwe_sk, 8 * p.n, cudaMemcpyDeviceToHost));
  if (glwe_sk)
    PNB_CUDA(cudaMemcpy(glwe_sk, K->glwe_sk, 8 * (size_t)p.k * p.N, cudaMemcpyDeviceToHost));
  if (bsk) PNB_CUDA(cudaMemcpy(bsk, K->bsk, 8 * K->bsk_words, cudaMemcpyDeviceToHost));
  if (ksk) {
    const size_t rows = (size_t)p.k * p.N * p.ks_level;
    PNB_CUDA(cudaMemcpy2D(ksk, 8 * (size_t)(p.n + 1), K->ksk, 8 * (size_t)K->ksk_row,
                          8 * (size_t)(p.n + 1), rows, cudaMemcpyDeviceToHost));
  }
  return PNB_OK;
}

int pnb_encrypt_lwe(const pnb_keys* K, const int64_t* messages_dev, uint64_t delta,
                    uint64_t seed, uint64_t first_index, uint64_t* ct_dev, int count,
                    void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!messages_dev || !ct_dev))) {
    set_error("encrypt: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  if ((rc = check_secret(K, false))) return rc;
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return encrypt_lwe(K, messages_dev, delta, seed, first_index, ct_dev, count,
                     (cudaStream_t)stream);
}

int pnb_phase_lwe(const pnb_keys* K, const uint64_t* ct_dev, uint64_t* phase_dev, int count,
                  int small_key, void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!ct_dev || !phase_dev))) {
    set_error("phase: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  if ((rc = check_secret(K, small_key != 0))) return rc;
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return phase_lwe(K, ct_dev, phase_dev, count, small_key, (cudaStream_t)stream);
}

int pnb_test_vector(const pnb_keys* K, const uint64_t* lut_host, int lut_len,
                    uint64_t delta_out, uint64_t* tv_dev, void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (!lut_host || !tv_dev) { set_error("test_vector: NULL buffer"); return PNB_ERR_INVALID; }
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return test_vector(K, lut_host, lut_len, delta_out, tv_dev, (cudaStream_t)stream);
}

size_t pnb_keyswitch_workspace_bytes(const pnb_keys* K, int count) {
  if (!K || count <= 0) return 0;
  return ks_tc_workspace_bytes(K->p, count);
}

int pnb_keyswitch(const pnb_keys* K, const uint64_t* in_dev, uint64_t* out_dev, int count,
                  void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!in_dev || !out_dev))) {
    set_error("keyswitch: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  if (workspace && (workspace_bytes < ks_tc_workspace_bytes(K->p, count) ||
                    (uintptr_t)workspace % 256 != 0)) {
    set_error("keyswitch: workspace must be 256-byte aligned and hold %zu bytes (got %zu)",
              ks_tc_workspace_bytes(K->p, count), workspace_bytes);
    return PNB_ERR_INVALID;
  }
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return keyswitch_launch(K, in_dev, out_dev, count, workspace, (cudaStream_t)stream);
}

int pnb_blind_rotate(const pnb_keys* K, const uint64_t* tv_dev, const uint64_t* small_dev,
                     uint64_t* out_dev, int count, void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!tv_dev || !small_dev || !out_dev))) {
    set_error("blind_rotate: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return blind_rotate_launch(K, tv_dev, small_dev, out_dev, count, (cudaStream_t)stream);
}

size_t pnb_pbs_workspace_bytes(const pnb_keys* K, int count) {
  return pbs_workspace_bytes(K, count);
}

int pnb_pbs_batch(const pnb_keys* K, const uint64_t* tv_dev, const uint64_t* in_dev,
                  uint64_t* out_dev, int count, void* workspace, size_t workspace_bytes,
                  void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!tv_dev || !in_dev || !out_dev))) {
    set_error("pbs: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  if (count > 0 && in_dev == out_dev) {
    set_error("pbs: input and output batches may not alias");
    return PNB_ERR_INVALID;
  }
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return pbs_batch(K, tv_dev, in_dev, out_dev, count, workspace, workspace_bytes,
                   (cudaStream_t)stream);
}

int pnb_pbs_batch_noalloc(const pnb_keys* K, const uint64_t* tv_dev, const uint64_t* in_dev,
                          uint64_t* out_dev, int count, void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!tv_dev || !in_dev || !out_dev))) {
    set_error("pbs_noalloc: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  if (count > 0 && in_dev == out_dev) {
    set_error("pbs_noalloc: input and output batches may not alias");
    return PNB_ERR_INVALID;
  }
  if (count == 0) return PNB_OK;
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return pbs_batch_noalloc(K, tv_dev, in_dev, out_dev, count, (cudaStream_t)stream);
}

int pnb_radix_merge(const pnb_keys* K, const uint64_t* blocks_dev, int num_blocks, int count,
                    int is_signed, uint64_t delta_out, uint64_t* out_dev, void* stream) {
  int rc = check_keys(K);
  if (rc) return rc;
  if (count < 0 || (count > 0 && (!blocks_dev || !out_dev))) {
    set_error("radix_merge: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  DeviceGuard g(K->device);
  if (g.rc) return g.rc;
  return radix_merge(K, blocks_dev, num_blocks, count, is_signed != 0, delta_out, out_dev,
                     (cudaStream_t)stream);
}

int pnb_lwe_contract(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta, int M, int K,
                     const uint64_t* X_dev, uint64_t* Y_dev, int batch, int lwe_len,
                     void* stream) {
  if (batch > 0 && (!W_dev || !X_dev || !Y_dev)) {
    set_error("contract: NULL buffer");
    return PNB_ERR_INVALID;
  }
  return lwe_contract_tc(W_dev, bias_dev, delta, M, K, X_dev, Y_dev, batch, lwe_len,
                         (cudaStream_t)stream);
}

int pnb_lwe_contract_gather(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta, int M,
                            int K, const uint64_t* X_dev, const int32_t* index_dev, int groups,
                            uint64_t* Y_dev, int lwe_len, void* stream) {
  if (groups > 0 && (!W_dev || !X_dev || !index_dev || !Y_dev)) {
    set_error("contract_gather: NULL buffer");
    return PNB_ERR_INVALID;
  }
  return lwe_contract_gather(W_dev, bias_dev, delta, M, K, X_dev, index_dev, groups, Y_dev,
                             lwe_len, (cudaStream_t)stream);
}

int pnb_lwe_contract_ld(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta, int M,
                        int K, const uint64_t* X_dev, int ldx, uint64_t* Y_dev, int ldy,
                        int batch, int lwe_len, void* stream) {
  if (batch > 0 && (!W_dev || !X_dev || !Y_dev)) {
    set_error("contract: NULL buffer");
    return PNB_ERR_INVALID;
  }
  if (ldx <= 0 || ldy <= 0) {
    set_error("contract: row pitches must be positive (got %d, %d)", ldx, ldy);
    return PNB_ERR_INVALID;
  }
  return lwe_contract_tc(W_dev, bias_dev, delta, M, K, X_dev, Y_dev, batch, lwe_len,
                         (cudaStream_t)stream, ldx, ldy);
}

int pnb_lwe_contract_gather_ld(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta,
                               int M, int K, const uint64_t* X_dev, int ldx,
                               const int32_t* index_dev, int groups, uint64_t* Y_dev, int ldy,
                               int lwe_len, void* stream) {
  if (groups > 0 && (!W_dev || !X_dev || !index_dev || !Y_dev)) {
    set_error("contract_gather: NULL buffer");
    return PNB_ERR_INVALID;
  }
  if (ldx <= 0 || ldy <= 0) {
    set_error("contract_gather: row pitches must be positive (got %d, %d)", ldx, ldy);
    return PNB_ERR_INVALID;
  }
  return lwe_contract_gather_placed(W_dev, bias_dev, delta, M, K, X_dev, index_dev, groups,
                                    Y_dev, lwe_len, 0, (cudaStream_t)stream, ldx, ldy);
}

int pnb_fft_negacyclic_mul(int device, int N, const int64_t* a_dev, const uint64_t* b_dev,
                           uint64_t* out_dev, int count, void* stream) {
  if (count < 0 || (count > 0 && (!a_dev || !b_dev || !out_dev))) {
    set_error("fft_mul: bad buffers or count %d", count);
    return PNB_ERR_INVALID;
  }
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  return fft_negacyclic_mul(N, a_dev, b_dev, out_dev, count, (cudaStream_t)stream);
}

int pnb_device_status(int device, int* status_out) {
  if (!status_out) { set_error("status_out is NULL"); return PNB_ERR_INVALID; }
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  int a = 0, b = 0, c = 0;
  int rc = tc_status_read_and_clear(&a);
  if (rc) return rc;
  rc = br_status_read_and_clear(&b);
  if (rc) return rc;
  rc = ct_status_read_and_clear(&c);
  if (rc) return rc;
  *status_out = a ? a : (b ? 16 + b : (c ? 32 + c : 0));
  return PNB_OK;
}

int pnb_measure_fp64_peak(int device, double* tflops_out) {
  if (!tflops_out) { set_error("tflops_out is NULL"); return PNB_ERR_INVALID; }
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  return measure_fp64_peak(tflops_out);
}

int pnb_wait_probe(int device, unsigned polls, int* warps_gave_up_out) {
  if (!warps_gave_up_out) { set_error("warps_gave_up_out is NULL"); return PNB_ERR_INVALID; }
  if (polls < 1 || polls > (1u << 24)) {
    set_error("wait probe: polls must be in 1..2^24 (got %u)", polls);
    return PNB_ERR_INVALID;
  }
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  return wait_probe(polls, warps_gave_up_out);
}

}  // extern "C"
