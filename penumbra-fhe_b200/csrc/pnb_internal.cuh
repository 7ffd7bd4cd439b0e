// pnb_internal.cuh -- shared device code for the Penumbra-FHE B200 kernels.
//
// Torus elements are u64 (ciphertext modulus 2^64).  An LWE ciphertext of dimension d is d+1
// u64 words, body last.  A GLWE ciphertext of dimension k over Z[X]/(X^N+1) is (k+1)*N words,
// body polynomial last.  These are the layouts the reference reaches through tfhe 1.6.3
// (runtime/src/ops/mod.rs:58 SignedRadixCiphertext blocks are shortint LWE ciphertexts).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/penumbra_b200.h"

namespace pnb {

// ------------------------------------------------------------------------------------------
// Error reporting (thread-local last-error string, integer status codes).
// ------------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

#define PNB_CUDA(call)                                                     \
  do {                                                                     \
    cudaError_t _e = (call);                                               \
    if (_e != cudaSuccess) return ::pnb::cuda_status(_e, #call);           \
  } while (0)

#define PNB_CHECK_LAUNCH(what)                                             \
  do {                                                                     \
    cudaError_t _e = cudaGetLastError();                                   \
    if (_e != cudaSuccess) return ::pnb::cuda_status(_e, what);            \
  } while (0)

// ------------------------------------------------------------------------------------------
// ChaCha20 keystream (original 64-bit nonce / 64-bit counter layout) keyed by a 64-bit seed.
// Word w of the stream (domain, index) is word (index & 7) of block (index >> 3).
// ------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t rotl32(uint32_t v, int c) {
  return (v << c) | (v >> (32 - c));
}

#define PNB_QR(a, b, c, d)          \
  a += b; d ^= a; d = rotl32(d, 16); \
  c += d; b ^= c; b = rotl32(b, 12); \
  a += b; d ^= a; d = rotl32(d, 8);  \
  c += d; b ^= c; b = rotl32(b, 7);

__host__ __device__ __forceinline__ void chacha20_block(uint64_t seed, uint64_t nonce,
                                                        uint64_t counter, uint32_t out[16]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    (uint32_t)seed, (uint32_t)(seed >> 32), 0x50454e55u, 0x4d425241u,
                    0x2d464845u, 0x2d423230u, 0x30000000u, 0x00000001u,
                    (uint32_t)counter, (uint32_t)(counter >> 32),
                    (uint32_t)nonce, (uint32_t)(nonce >> 32)};
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = s[i];
#pragma unroll 1
  for (int r = 0; r < 10; ++r) {
    PNB_QR(x[0], x[4], x[8], x[12]) PNB_QR(x[1], x[5], x[9], x[13])
    PNB_QR(x[2], x[6], x[10], x[14]) PNB_QR(x[3], x[7], x[11], x[15])
    PNB_QR(x[0], x[5], x[10], x[15]) PNB_QR(x[1], x[6], x[11], x[12])
    PNB_QR(x[2], x[7], x[8], x[13]) PNB_QR(x[3], x[4], x[9], x[14])
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

__host__ __device__ __forceinline__ uint64_t rand_word(uint64_t seed, uint64_t domain,
                                                       uint64_t index) {
  uint32_t blk[16];
  chacha20_block(seed, domain, index >> 3, blk);
  int w = (int)(index & 7);
  uint64_t lo = 0, hi = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    if (t == w) { lo = blk[2 * t]; hi = blk[2 * t + 1]; }
  }
  return lo | (hi << 32);
}

// Keystream domains (ChaCha20 nonces) -- one independent stream per key component.
enum : uint64_t {
  DOM_LWE_SK = 1, DOM_GLWE_SK = 2, DOM_BSK_MASK = 3, DOM_BSK_NOISE = 4,
  DOM_KSK_MASK = 5, DOM_KSK_NOISE = 6, DOM_ENC_MASK = 7, DOM_ENC_NOISE = 8
};

// ------------------------------------------------------------------------------------------
// Signed gadget decomposition with round-to-nearest.  digits[j] multiplies 2^(64-beta(j+1)),
// each digit in [-B/2, B/2).  Requires beta*level < 64.
// ------------------------------------------------------------------------------------------
template <int LEVEL>
__device__ __forceinline__ void decompose(uint64_t a, int beta, int64_t (&digits)[LEVEL]) {
  const int total = beta * LEVEL;
  uint64_t st = (a >> (64 - total)) + ((a >> (63 - total)) & 1u);
  const uint64_t mask = (1ull << beta) - 1, half = 1ull << (beta - 1);
#pragma unroll
  for (int j = LEVEL - 1; j >= 0; --j) {
    uint64_t d = st & mask;
    st >>= beta;
    bool neg = d >= half;
    digits[j] = neg ? (int64_t)d - (int64_t)(1ull << beta) : (int64_t)d;
    st += neg ? 1u : 0u;
  }
}

__device__ __forceinline__ int modswitch(uint64_t x, int log2_2N) {
  uint64_t r = ((x >> (63 - log2_2N)) + 1) >> 1;
  return (int)(r & ((1ull << log2_2N) - 1));
}

__host__ __device__ __forceinline__ int ilog2i(int v) {
  int r = 0;
  while ((1 << r) < v) ++r;
  return r;
}

// ------------------------------------------------------------------------------------------
// f64 <-> torus conversion.
// ------------------------------------------------------------------------------------------
// Exact double of a signed integer |d| < 2^51 without the conversion unit: add to the bits of
// 1.5 * 2^52 and subtract that constant on the FP64 pipe.
__device__ __forceinline__ double small_int_to_f64(int64_t d) {
  const double magic = 6755399441055744.0;  // 1.5 * 2^52
  return __longlong_as_double(__double_as_longlong(magic) + d) - magic;
}

// Round an integer-valued double of any magnitude to the nearest integer modulo 2^64.  For
// |v| >= 2^52 the value is already an integer and its low 64 bits come straight from the
// mantissa; below that the conversion unit rounds it.
__device__ __forceinline__ uint64_t f64_to_torus(double v) {
  const long long bits = __double_as_longlong(v);
  const int e = (int)((bits >> 52) & 0x7ff) - 1075;  // v = mant * 2^e
  if (e < 0) return (uint64_t)__double2ll_rn(v);
  const uint64_t mant = ((uint64_t)bits & 0x000fffffffffffffull) | 0x0010000000000000ull;
  const uint64_t mag = (e < 64) ? (mant << e) : 0ull;
  return (bits < 0) ? (uint64_t)0 - mag : mag;
}

}  // namespace pnb
