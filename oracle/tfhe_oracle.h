/*
 * tfhe_oracle.h -- CPU restatement of the TFHE arithmetic behind Penumbra-FHE's encrypted
 * evaluation path.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and the CPU
 * baseline leg of the benchmark link this; the product library never does.
 *
 * The reference (Penumbra-FHE) delegates every ciphertext operation to the crates.io
 * dependency `tfhe` 1.6.3 (runtime/Cargo.toml:20, runtime/Cargo.lock), which is not vendored.
 * Its call sites are runtime/src/keys.rs:55 (gen_keys_radix), runtime/src/encrypt.rs:21,35,44,
 * runtime/src/ops/activation.rs:104,115 and runtime/src/ops/requant.rs:193,232
 * (generate_lookup_table / apply_lookup_table = keyswitch + PBS), runtime/src/ops/linear.rs:66-73
 * (scalar_mul / add over ciphertexts).  This file restates the published TFHE/CGGI algorithms
 * (Chillotti-Gama-Georgieva-Izabachene, J. Cryptology 2020; Joye, "Guide to FHE over the
 * discretized torus", 2021) that those calls execute, with the parameter layout of the
 * shortint "KS_PBS" order: client ciphertexts live under the big key (dimension k*N), are
 * keyswitched to the small key (dimension n), bootstrapped, and come back under the big key.
 *
 * Parity status: ciphertext bits, key bits and CSPRNG streams of tfhe-rs are not pinned (the
 * crate is absent and the reference serialises nothing); decrypted values are pinned by the
 * reference's own golden tests (runtime/tests/hello_fhe.rs:50-67 LUT sweep, golden_requant*.rs
 * sweeps, examples fixtures).  The integer parts here (keys, keyswitch, contraction, exact blind
 * rotation) define bit-exact results for the CUDA path; the f64-FFT blind rotation restates the
 * approximate FFT product tfhe-rs uses and serves as the CPU baseline.
 */
#ifndef PNB_TFHE_ORACLE_H
#define PNB_TFHE_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t n;            /* small LWE dimension */
  int32_t k;            /* GLWE dimension */
  int32_t N;            /* polynomial size */
  int32_t pbs_base_log; /* bootstrapping gadget base log */
  int32_t pbs_level;
  int32_t ks_base_log;  /* keyswitch gadget base log */
  int32_t ks_level;
  int32_t msg_bits;     /* message bits per block */
  int32_t carry_bits;   /* carry bits per block */
  int32_t _pad;
  double lwe_std;       /* noise std of small-key LWE (fraction of the torus) */
  double glwe_std;      /* noise std of GLWE / big-key LWE (fraction of the torus) */
} orc_params;

/* CSPRNG: ChaCha20 (64-bit nonce, 64-bit block counter) keyed by a 64-bit seed. */
uint64_t orc_rand_word(uint64_t seed, uint64_t domain, uint64_t index);
void orc_chacha20_block(uint64_t seed, uint64_t nonce, uint64_t counter, uint32_t out[16]);
void orc_chacha20_block_key(const uint32_t key[8], uint64_t nonce, uint64_t counter,
                            uint32_t out[16]);
double orc_ln(double u);
double orc_cos2pi(double u);
int64_t orc_gaussian(uint64_t seed, uint64_t domain, uint64_t index, double sigma_abs);

/* Key material (all u64 arrays, caller-allocated). */
void orc_secret_keys(const orc_params* p, uint64_t seed, uint64_t* lwe_sk, uint64_t* glwe_sk);
size_t orc_bsk_words(const orc_params* p);
size_t orc_ksk_words(const orc_params* p);
void orc_bsk_gen(const orc_params* p, uint64_t seed, const uint64_t* lwe_sk,
                 const uint64_t* glwe_sk, uint64_t* bsk);
void orc_ksk_gen(const orc_params* p, uint64_t seed, const uint64_t* glwe_sk,
                 const uint64_t* lwe_sk, uint64_t* ksk);

/* LWE helpers. ct has dim+1 words, body last. */
void orc_lwe_encrypt(int dim, const uint64_t* key, uint64_t plaintext, uint64_t seed,
                     uint64_t index, double sigma, uint64_t* ct);
uint64_t orc_lwe_phase(int dim, const uint64_t* key, const uint64_t* ct);
uint64_t orc_delta(const orc_params* p);
uint64_t orc_decode(const orc_params* p, uint64_t phase); /* round(phase/delta) mod 2*msg_space */

/* Keyswitch big (k*N) -> small (n). */
void orc_keyswitch(const orc_params* p, const uint64_t* ksk, const uint64_t* in, uint64_t* out);

/* Programmable bootstrap pieces. */
void orc_test_vector(const orc_params* p, const uint64_t* lut, int lut_len, uint64_t delta_out,
                     uint64_t* tv);
void orc_negacyclic_mul(int N, const uint64_t* a, const uint64_t* b, uint64_t* out);
void orc_blind_rotate_exact(const orc_params* p, const uint64_t* bsk, const uint64_t* ct_small,
                            const uint64_t* tv, uint64_t* glwe);
void orc_sample_extract(const orc_params* p, const uint64_t* glwe, uint64_t* lwe_big);
void orc_pbs_exact(const orc_params* p, const uint64_t* bsk, const uint64_t* ksk,
                   const uint64_t* tv, const uint64_t* in, uint64_t* out, int count,
                   int threads);

/* f64 negacyclic-FFT bootstrap (approximate product, as tfhe-rs computes it). */
size_t orc_fourier_bsk_doubles(const orc_params* p);
void orc_bsk_to_fourier(const orc_params* p, const uint64_t* bsk, double* fbsk);
void orc_pbs_fft(const orc_params* p, const double* fbsk, const uint64_t* ksk,
                 const uint64_t* tv, const uint64_t* in, uint64_t* out, int count, int threads);

/* Ciphertext x cleartext-weight contraction:
 *   Y[b][j][c] = sum_i W[j][i] * X[b][i][c]  (mod 2^64), plus bias[j]*delta on the body column.
 * X is [batch][K][lwe_len], Y is [batch][M][lwe_len], W is [M][K] int64, bias may be NULL. */
void orc_contract(const int64_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                  const uint64_t* X, uint64_t* Y, int batch, int lwe_len, int threads);

#ifdef __cplusplus
}
#endif
#endif
