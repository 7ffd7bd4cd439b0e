// pnb_keys.h -- the opaque key set behind pnb_keys* and the internal launch entry points.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/penumbra_b200.h"

struct pnb_keys {
  int device;
  pnb_params p;
  uint64_t seed;
  uint64_t* lwe_sk;    // [n]            small secret key (client side, harness only)
  uint64_t* glwe_sk;   // [k*N]          GLWE secret key = big LWE key (client side)
  uint64_t* bsk;       // [n][(k+1)l][k+1][N] standard-domain bootstrapping key
  double2* fbsk;       // [n][(k+1)l][k+1][N/2] Fourier bootstrapping key (permuted spectrum)
  uint64_t* ksk;       // [k*N][ks_level][ksk_row] keyswitching key, rows padded to 16 bytes
  int ksk_row;         // words per keyswitching-key row (n+1 rounded up to even)
  size_t bsk_words;
  size_t fbsk_elems;
  size_t ksk_words;
};

namespace pnb {
int keygen_device(pnb_keys* K, cudaStream_t st);
int bsk_to_fourier(const uint64_t* bsk_dev, double2* fbsk_dev, int polys, cudaStream_t st);
// N = 8192 (pbs8k.cu): Fourier conversion into the 4096-point transform's spectral order, and the
// blind rotation + sample extraction of the 6-bit set.
int bsk_to_fourier_8k(const uint64_t* bsk_dev, double2* fbsk_dev, int polys, cudaStream_t st);
bool br8k_supported(const pnb_params& p);
int fft_negacyclic_mul_8k(const int64_t* a, const uint64_t* b, uint64_t* out, int count,
                          cudaStream_t st);
int blind_rotate_8k(const pnb_keys* K, const uint64_t* tvs, const int32_t* tv_idx, int period,
                    int first, const uint64_t* small, uint64_t* out, int out_ld, int count,
                    cudaStream_t st);
// Row pitches in words (`*_ld`, 0 = contiguous rows of the natural length) let the graph
// evaluator keep its ciphertext rows 16-byte aligned.
int keyswitch_launch(const pnb_keys* K, const uint64_t* in, uint64_t* out, int count,
                     void* digits, cudaStream_t st, int in_ld = 0);
// Per-ciphertext test vectors: ciphertext c starts from tvs + tv_idx[(first + c) % period] * N.
int blind_rotate_sel(const pnb_keys* K, const uint64_t* tvs, const int32_t* tv_idx, int period,
                     int first, const uint64_t* small, uint64_t* out, int count, cudaStream_t st,
                     int out_ld = 0);
int blind_rotate_launch(const pnb_keys* K, const uint64_t* tv, const uint64_t* small,
                        uint64_t* out, int count, cudaStream_t st);
size_t pbs_workspace_bytes(const pnb_keys* K, int count);
int pbs_batch(const pnb_keys* K, const uint64_t* tv, const uint64_t* in, uint64_t* out,
              int count, void* ws, size_t ws_bytes, cudaStream_t st);
int test_vector(const pnb_keys* K, const uint64_t* lut_host, int lut_len, uint64_t delta_out,
                uint64_t* tv, cudaStream_t st);
// Merge [count][nb] radix-block ciphertexts into [count] wide ciphertexts (radix.cu).
int radix_merge(const pnb_keys* K, const uint64_t* blocks, int nb, int count, bool is_signed,
                uint64_t delta_out, uint64_t* out, cudaStream_t st);
void radix_merge_lut(int msg_bits, int carry_bits, int nb, int i, bool is_signed, uint64_t* lut);
int fft_negacyclic_mul(int N, const int64_t* a, const uint64_t* b, uint64_t* out, int count,
                       cudaStream_t st);
int encrypt_lwe(const pnb_keys* K, const int64_t* msg, uint64_t delta, uint64_t seed,
                uint64_t first, uint64_t* ct, int count, cudaStream_t st);
int phase_lwe(const pnb_keys* K, const uint64_t* ct, uint64_t* phase, int count, int small,
              cudaStream_t st);
int measure_fp64_peak(double* tflops);
int wait_probe(uint32_t polls, int* warps_gave_up);
int lwe_contract_tc(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                    const uint64_t* X, uint64_t* Y, int batch, int L, cudaStream_t st,
                    int ldx = 0, int ldy = 0);
// As lwe_contract_gather, with group g = b*P + p written to output row (b*M + m)*P + p
// (the channel-major [sample][channel][position] layout of a convolution); P = 0: [g][m].
int lwe_contract_gather_placed(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                               const uint64_t* X, const int32_t* idx, int G, uint64_t* Y, int L,
                               int P, cudaStream_t st, int ldx = 0, int ldy = 0);
int lwe_contract_gather(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                        const uint64_t* X, const int32_t* idx, int G, uint64_t* Y, int L,
                        cudaStream_t st);
int keyswitch_tc(const pnb_keys* K, const uint64_t* in, uint64_t* out, int count, void* digits,
                 cudaStream_t st, int in_ld = 0);
size_t ks_tc_workspace_bytes(const pnb_params& p, int count);
int tc_status_read_and_clear(int* out);
bool fft_tables_ready();
int pbs_batch_noalloc(const pnb_keys* K, const uint64_t* tv, const uint64_t* in, uint64_t* out,
                      int count, cudaStream_t st);
int br_status_read_and_clear(int* out);
int br8_status_read_and_clear(int* out);
int ct_status_read_and_clear(int* out);
}  // namespace pnb
