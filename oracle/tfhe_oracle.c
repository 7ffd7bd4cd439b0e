/*
 * tfhe_oracle.c -- CPU restatement of the TFHE arithmetic on Penumbra-FHE's encrypted path.
 * TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline); the product never links it.
 *
 * Algorithms restated from the published TFHE/CGGI construction that the reference reaches
 * through tfhe 1.6.3 (see tfhe_oracle.h for the call sites).  Every function here is written so
 * that its integer results are bit-exact definitions for the CUDA path:
 *   - ChaCha20 keystream (D. J. Bernstein, "ChaCha, a variant of Salsa20", 2008), original
 *     64-bit-nonce / 64-bit-counter layout;
 *   - Box-Muller Gaussian with a series ln / cos built only from +,-,*,/,sqrt,fma so that a
 *     CPU and a GPU evaluation produce identical doubles;
 *   - GLWE / GGSW / LWE key-switching-key generation (CGGI 2020, sec. 3-4);
 *   - signed gadget decomposition with round-to-nearest (Joye 2021, sec. 4.2);
 *   - keyswitch, modulus switch, CMux blind rotation, sample extraction (CGGI 2020, alg. 3-4);
 *   - an exact mod-2^64 negacyclic product (Karatsuba over wrapping u64) and the
 *     approximate f64 negacyclic FFT product ("folding" of the N-coefficient real polynomial
 *     into an N/2-point complex FFT with a 2N-th root twist).
 */
#include "tfhe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------ */
/* ChaCha20 keystream                                                                          */
/* ------------------------------------------------------------------------------------------ */
#define ROTL32(v, c) (((v) << (c)) | ((v) >> (32 - (c))))
#define QR(a, b, c, d)                                                                           \
  a += b; d ^= a; d = ROTL32(d, 16);                                                              \
  c += d; b ^= c; b = ROTL32(b, 12);                                                              \
  a += b; d ^= a; d = ROTL32(d, 8);                                                               \
  c += d; b ^= c; b = ROTL32(b, 7);

void orc_chacha20_block_key(const uint32_t key[8], uint64_t nonce, uint64_t counter,
                            uint32_t out[16]) {
  uint32_t s[16];
  s[0] = 0x61707865u; s[1] = 0x3320646eu; s[2] = 0x79622d32u; s[3] = 0x6b206574u;
  for (int i = 0; i < 8; ++i) s[4 + i] = key[i];
  s[12] = (uint32_t)counter; s[13] = (uint32_t)(counter >> 32);
  s[14] = (uint32_t)nonce; s[15] = (uint32_t)(nonce >> 32);
  uint32_t x[16];
  memcpy(x, s, sizeof(x));
  for (int r = 0; r < 10; ++r) {
    QR(x[0], x[4], x[8], x[12]) QR(x[1], x[5], x[9], x[13])
    QR(x[2], x[6], x[10], x[14]) QR(x[3], x[7], x[11], x[15])
    QR(x[0], x[5], x[10], x[15]) QR(x[1], x[6], x[11], x[12])
    QR(x[2], x[7], x[8], x[13]) QR(x[3], x[4], x[9], x[14])
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

/* 256-bit key: the 64-bit seed followed by a fixed, documented filler. */
void orc_chacha20_block(uint64_t seed, uint64_t nonce, uint64_t counter, uint32_t out[16]) {
  const uint32_t key[8] = {(uint32_t)seed, (uint32_t)(seed >> 32), 0x50454e55u, 0x4d425241u,
                           0x2d464845u, 0x2d423230u, 0x30000000u, 0x00000001u};
  orc_chacha20_block_key(key, nonce, counter, out);
}

uint64_t orc_rand_word(uint64_t seed, uint64_t domain, uint64_t index) {
  uint32_t blk[16];
  orc_chacha20_block(seed, domain, index >> 3, blk);
  int w = (int)(index & 7);
  return (uint64_t)blk[2 * w] | ((uint64_t)blk[2 * w + 1] << 32);
}

/* ------------------------------------------------------------------------------------------ */
/* Deterministic Gaussian: Box-Muller with series ln and cos (identical on CPU and GPU).      */
/* ------------------------------------------------------------------------------------------ */
static inline double bits_to_f64(uint64_t b) { double d; memcpy(&d, &b, 8); return d; }
static inline uint64_t f64_to_bits(double d) { uint64_t b; memcpy(&b, &d, 8); return b; }

/* ln(u) for normal u > 0: u = m 2^e, m in [sqrt(1/2), sqrt(2)], ln m = 2 atanh((m-1)/(m+1)). */
double orc_ln(double u) {
  uint64_t b = f64_to_bits(u);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  double m = bits_to_f64((b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL);
  if (m > 0x1.6a09e667f3bcdp+0) { m = m * 0.5; e += 1; }
  double s = (m - 1.0) / (m + 1.0);
  double s2 = s * s;
  double p = 0x1.642c8590b2164p-5;         /* 1/23 */
  p = fma(p, s2, 0x1.8618618618618p-5);    /* 1/21 */
  p = fma(p, s2, 0x1.af286bca1af28p-5);    /* 1/19 */
  p = fma(p, s2, 0x1.e1e1e1e1e1e1ep-5);    /* 1/17 */
  p = fma(p, s2, 0x1.1111111111111p-4);    /* 1/15 */
  p = fma(p, s2, 0x1.3b13b13b13b14p-4);    /* 1/13 */
  p = fma(p, s2, 0x1.745d1745d1746p-4);    /* 1/11 */
  p = fma(p, s2, 0x1.c71c71c71c71cp-4);    /* 1/9 */
  p = fma(p, s2, 0x1.2492492492492p-3);    /* 1/7 */
  p = fma(p, s2, 0x1.999999999999ap-3);    /* 1/5 */
  p = fma(p, s2, 0x1.5555555555555p-2);    /* 1/3 */
  p = fma(p, s2, 1.0);
  double t = s * p;
  t = t + t;
  return fma((double)e, 0x1.62e42fefa39efp-1, t);
}

/* cos(2 pi u) for u in [0, 1): fold to [0, 1/4], Taylor series of cos on [0, pi/2]. */
double orc_cos2pi(double u) {
  double t = u - rint(u);
  t = fabs(t);
  double sign = 1.0;
  if (t > 0.25) { t = 0.5 - t; sign = -1.0; }
  double x = t * 0x1.921fb54442d18p+2;
  double x2 = x * x;
  double p = 0x1.f2cf01972f578p-80;        /* 1/24! */
  p = fma(p, x2, -0x1.0ce396db7f853p-70);  /* -1/22! */
  p = fma(p, x2, 0x1.e542ba4020225p-62);   /* 1/20! */
  p = fma(p, x2, -0x1.6827863b97d97p-53);  /* -1/18! */
  p = fma(p, x2, 0x1.ae7f3e733b81fp-45);   /* 1/16! */
  p = fma(p, x2, -0x1.93974a8c07c9dp-37);  /* -1/14! */
  p = fma(p, x2, 0x1.1eed8eff8d898p-29);   /* 1/12! */
  p = fma(p, x2, -0x1.27e4fb7789f5cp-22);  /* -1/10! */
  p = fma(p, x2, 0x1.a01a01a01a01ap-16);   /* 1/8! */
  p = fma(p, x2, -0x1.6c16c16c16c17p-10);  /* -1/6! */
  p = fma(p, x2, 0x1.5555555555555p-5);    /* 1/4! */
  p = fma(p, x2, -0.5);
  p = fma(p, x2, 1.0);
  return sign * p;
}

/* One centred Gaussian sample of std sigma_abs (torus units), rounded to an integer.
 * Uses keystream words 2*index and 2*index+1 of the noise domain. */
int64_t orc_gaussian(uint64_t seed, uint64_t domain, uint64_t index, double sigma_abs) {
  uint64_t w1 = orc_rand_word(seed, domain, 2 * index);
  uint64_t w2 = orc_rand_word(seed, domain, 2 * index + 1);
  double u1 = (double)((w1 >> 11) + 1) * 0x1p-53; /* (0, 1] */
  double u2 = (double)(w2 >> 11) * 0x1p-53;       /* [0, 1) */
  double l = orc_ln(u1);
  double r = sqrt(-2.0 * l);
  double z = r * orc_cos2pi(u2);
  double v = z * sigma_abs;
  return (int64_t)llrint(v);
}

/* Keystream domains (ChaCha20 nonces). */
enum {
  DOM_LWE_SK = 1, DOM_GLWE_SK = 2, DOM_BSK_MASK = 3, DOM_BSK_NOISE = 4,
  DOM_KSK_MASK = 5, DOM_KSK_NOISE = 6, DOM_ENC_MASK = 7, DOM_ENC_NOISE = 8
};

/* ------------------------------------------------------------------------------------------ */
/* Keys                                                                                        */
/* ------------------------------------------------------------------------------------------ */
void orc_secret_keys(const orc_params* p, uint64_t seed, uint64_t* lwe_sk, uint64_t* glwe_sk) {
  for (int i = 0; i < p->n; ++i) lwe_sk[i] = orc_rand_word(seed, DOM_LWE_SK, (uint64_t)i) & 1u;
  for (int i = 0; i < p->k * p->N; ++i)
    glwe_sk[i] = orc_rand_word(seed, DOM_GLWE_SK, (uint64_t)i) & 1u;
}

size_t orc_bsk_words(const orc_params* p) {
  return (size_t)p->n * (p->k + 1) * p->pbs_level * (p->k + 1) * p->N;
}
size_t orc_ksk_words(const orc_params* p) {
  return (size_t)p->k * p->N * p->ks_level * (p->n + 1);
}

/* out += a * s (negacyclic) for a binary polynomial s. */
static void negacyclic_mac_binary(int N, const uint64_t* a, const uint64_t* s, uint64_t* out) {
  for (int j = 0; j < N; ++j) {
    if (!s[j]) continue;
    /* X^j * a: coefficient t receives a[t-j] (t >= j) or -a[t-j+N] (t < j). */
    for (int t = 0; t < j; ++t) out[t] -= a[t - j + N];
    for (int t = j; t < N; ++t) out[t] += a[t - j];
  }
}

void orc_bsk_gen(const orc_params* p, uint64_t seed, const uint64_t* lwe_sk,
                 const uint64_t* glwe_sk, uint64_t* bsk) {
  const int N = p->N, k = p->k, l = p->pbs_level, rows = (k + 1) * l;
  const double sig = p->glwe_std * 0x1p64;
#pragma omp parallel for schedule(dynamic)
  for (int i = 0; i < p->n; ++i) {
    for (int r = 0; r < rows; ++r) {
      uint64_t* g = bsk + ((size_t)i * rows + r) * (k + 1) * N;
      uint64_t* body = g + (size_t)k * N;
      for (int t = 0; t < N; ++t) {
        uint64_t idx = ((uint64_t)i * rows + r) * N + t;
        body[t] = (uint64_t)orc_gaussian(seed, DOM_BSK_NOISE, idx, sig);
      }
      for (int c = 0; c < k; ++c) {
        uint64_t* a = g + (size_t)c * N;
        for (int t = 0; t < N; ++t) {
          uint64_t idx = (((uint64_t)i * rows + r) * k + c) * N + t;
          a[t] = orc_rand_word(seed, DOM_BSK_MASK, idx);
        }
        negacyclic_mac_binary(N, a, glwe_sk + (size_t)c * N, body);
      }
      int comp = r / l, lev = r % l;
      uint64_t gadget = lwe_sk[i] << (64 - p->pbs_base_log * (lev + 1));
      g[(size_t)comp * N] += gadget;
    }
  }
}

void orc_ksk_gen(const orc_params* p, uint64_t seed, const uint64_t* glwe_sk,
                 const uint64_t* lwe_sk, uint64_t* ksk) {
  const int n = p->n, big = p->k * p->N, L = p->ks_level;
  const double sig = p->lwe_std * 0x1p64;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < big; ++i) {
    for (int j = 0; j < L; ++j) {
      uint64_t* ct = ksk + ((size_t)i * L + j) * (n + 1);
      uint64_t b = 0;
      for (int t = 0; t < n; ++t) {
        uint64_t a = orc_rand_word(seed, DOM_KSK_MASK, ((uint64_t)i * L + j) * n + t);
        ct[t] = a;
        b += a * lwe_sk[t];
      }
      b += (uint64_t)orc_gaussian(seed, DOM_KSK_NOISE, (uint64_t)i * L + j, sig);
      b += glwe_sk[i] << (64 - p->ks_base_log * (j + 1));
      ct[n] = b;
    }
  }
}

/* ------------------------------------------------------------------------------------------ */
/* LWE                                                                                         */
/* ------------------------------------------------------------------------------------------ */
void orc_lwe_encrypt(int dim, const uint64_t* key, uint64_t plaintext, uint64_t seed,
                     uint64_t index, double sigma, uint64_t* ct) {
  uint64_t b = 0;
  for (int t = 0; t < dim; ++t) {
    uint64_t a = orc_rand_word(seed, DOM_ENC_MASK, index * (uint64_t)dim + t);
    ct[t] = a;
    b += a * key[t];
  }
  b += (uint64_t)orc_gaussian(seed, DOM_ENC_NOISE, index, sigma * 0x1p64);
  ct[dim] = b + plaintext;
}

uint64_t orc_lwe_phase(int dim, const uint64_t* key, const uint64_t* ct) {
  uint64_t s = 0;
  for (int t = 0; t < dim; ++t) s += ct[t] * key[t];
  return ct[dim] - s;
}

uint64_t orc_delta(const orc_params* p) {
  return 1ULL << (63 - p->msg_bits - p->carry_bits);
}

uint64_t orc_decode(const orc_params* p, uint64_t phase) {
  int shift = 63 - p->msg_bits - p->carry_bits;
  uint64_t r = (phase >> (shift - 1)) + 1; /* round to nearest multiple of delta */
  r >>= 1;
  return r & ((2ULL << (p->msg_bits + p->carry_bits)) - 1);
}

/* Signed gadget decomposition with round-to-nearest: digits[j] multiplies 2^(64-beta(j+1)),
 * each digit in [-B/2, B/2). */
static inline void decompose(uint64_t a, int beta, int level, int64_t* digits) {
  int total = beta * level;
  uint64_t st = (a >> (64 - total)) + ((a >> (63 - total)) & 1u);
  uint64_t mask = (1ULL << beta) - 1, half = 1ULL << (beta - 1);
  for (int j = level - 1; j >= 0; --j) {
    uint64_t d = st & mask;
    st >>= beta;
    if (d >= half) { digits[j] = (int64_t)d - (int64_t)(1ULL << beta); st += 1; }
    else digits[j] = (int64_t)d;
  }
}

void orc_keyswitch(const orc_params* p, const uint64_t* ksk, const uint64_t* in, uint64_t* out) {
  const int n = p->n, big = p->k * p->N, L = p->ks_level;
  for (int t = 0; t < n; ++t) out[t] = 0;
  out[n] = in[big];
  int64_t dig[64];
  for (int i = 0; i < big; ++i) {
    decompose(in[i], p->ks_base_log, L, dig);
    for (int j = 0; j < L; ++j) {
      if (!dig[j]) continue;
      const uint64_t* row = ksk + ((size_t)i * L + j) * (n + 1);
      uint64_t d = (uint64_t)dig[j];
      for (int t = 0; t <= n; ++t) out[t] -= d * row[t];
    }
  }
}

/* ------------------------------------------------------------------------------------------ */
/* Blind rotation                                                                              */
/* ------------------------------------------------------------------------------------------ */
void orc_test_vector(const orc_params* p, const uint64_t* lut, int lut_len, uint64_t delta_out,
                     uint64_t* tv) {
  const int N = p->N, box = N / lut_len, half = box / 2;
  for (int j = 0; j < N; ++j) {
    int m = (j + half) / box;
    tv[j] = (m < lut_len) ? lut[m] * delta_out : (uint64_t)0 - lut[m - lut_len] * delta_out;
  }
}

static inline int modswitch(uint64_t x, int log2_2N) {
  uint64_t r = ((x >> (63 - log2_2N)) + 1) >> 1;
  return (int)(r & ((1ULL << log2_2N) - 1));
}

static inline int ilog2(int v) { int r = 0; while ((1 << r) < v) ++r; return r; }

/* out = X^r * in (negacyclic), r in [0, 2N). */
static void rotate(int N, const uint64_t* in, int r, uint64_t* out) {
  for (int t = 0; t < N; ++t) {
    int s = t - r;
    int neg = 0;
    while (s < 0) { s += N; neg ^= 1; }
    out[t] = neg ? (uint64_t)0 - in[s] : in[s];
  }
}

static void kara(const uint64_t* a, const uint64_t* b, uint64_t* r, int n, uint64_t* tmp) {
  if (n <= 32) {
    for (int i = 0; i < 2 * n; ++i) r[i] = 0;
    for (int i = 0; i < n; ++i) {
      uint64_t ai = a[i];
      for (int j = 0; j < n; ++j) r[i + j] += ai * b[j];
    }
    return;
  }
  int h = n / 2;
  kara(a, b, r, h, tmp);
  kara(a + h, b + h, r + n, h, tmp);
  uint64_t *t1 = tmp, *t2 = tmp + h, *t3 = tmp + 2 * h, *nx = tmp + 4 * h;
  for (int i = 0; i < h; ++i) { t1[i] = a[i] + a[i + h]; t2[i] = b[i] + b[i + h]; }
  kara(t1, t2, t3, h, nx);
  for (int i = 0; i < 2 * h; ++i) t3[i] -= r[i] + r[n + i];
  for (int i = 0; i < 2 * h; ++i) r[h + i] += t3[i];
}

/* Exact negacyclic product mod (X^N + 1, 2^64). */
void orc_negacyclic_mul(int N, const uint64_t* a, const uint64_t* b, uint64_t* out) {
  uint64_t* full = (uint64_t*)malloc(sizeof(uint64_t) * 2 * N);
  uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * 4 * N);
  kara(a, b, full, N, tmp);
  for (int j = 0; j < N; ++j) out[j] = full[j] - full[j + N];
  free(full);
  free(tmp);
}

void orc_blind_rotate_exact(const orc_params* p, const uint64_t* bsk, const uint64_t* ct_small,
                            const uint64_t* tv, uint64_t* glwe) {
  const int N = p->N, k = p->k, l = p->pbs_level, rows = (k + 1) * l, n = p->n;
  const int lg = ilog2(2 * N);
  int bt = modswitch(ct_small[n], lg);
  for (int c = 0; c < k; ++c) memset(glwe + (size_t)c * N, 0, sizeof(uint64_t) * N);
  rotate(N, tv, (2 * N - bt) % (2 * N), glwe + (size_t)k * N);
  uint64_t* rot = (uint64_t*)malloc(sizeof(uint64_t) * N);
  uint64_t* dig = (uint64_t*)malloc(sizeof(uint64_t) * rows * N);
  uint64_t* prod = (uint64_t*)malloc(sizeof(uint64_t) * N);
  int64_t dd[64];
  for (int i = 0; i < n; ++i) {
    int ai = modswitch(ct_small[i], lg);
    if (ai == 0) continue;
    for (int c = 0; c <= k; ++c) {
      rotate(N, glwe + (size_t)c * N, ai, rot);
      for (int t = 0; t < N; ++t) {
        decompose(rot[t] - glwe[(size_t)c * N + t], p->pbs_base_log, l, dd);
        for (int j = 0; j < l; ++j) dig[((size_t)c * l + j) * N + t] = (uint64_t)dd[j];
      }
    }
    const uint64_t* ggsw = bsk + (size_t)i * rows * (k + 1) * N;
    for (int r = 0; r < rows; ++r) {
      for (int c = 0; c <= k; ++c) {
        orc_negacyclic_mul(N, dig + (size_t)r * N, ggsw + ((size_t)r * (k + 1) + c) * N, prod);
        for (int t = 0; t < N; ++t) glwe[(size_t)c * N + t] += prod[t];
      }
    }
  }
  free(rot);
  free(dig);
  free(prod);
}

void orc_sample_extract(const orc_params* p, const uint64_t* glwe, uint64_t* lwe_big) {
  const int N = p->N, k = p->k;
  for (int c = 0; c < k; ++c) {
    const uint64_t* a = glwe + (size_t)c * N;
    lwe_big[(size_t)c * N] = a[0];
    for (int j = 1; j < N; ++j) lwe_big[(size_t)c * N + j] = (uint64_t)0 - a[N - j];
  }
  lwe_big[(size_t)k * N] = glwe[(size_t)k * N];
}

void orc_pbs_exact(const orc_params* p, const uint64_t* bsk, const uint64_t* ksk,
                   const uint64_t* tv, const uint64_t* in, uint64_t* out, int count,
                   int threads) {
  const int big = p->k * p->N;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for schedule(dynamic)
  for (int c = 0; c < count; ++c) {
    uint64_t* small = (uint64_t*)malloc(sizeof(uint64_t) * (p->n + 1));
    uint64_t* glwe = (uint64_t*)malloc(sizeof(uint64_t) * (p->k + 1) * p->N);
    orc_keyswitch(p, ksk, in + (size_t)c * (big + 1), small);
    orc_blind_rotate_exact(p, bsk, small, tv, glwe);
    orc_sample_extract(p, glwe, out + (size_t)c * (big + 1));
    free(small);
    free(glwe);
  }
}

/* ------------------------------------------------------------------------------------------ */
/* Approximate f64 negacyclic FFT product                                                      */
/* ------------------------------------------------------------------------------------------ */
typedef struct { double re, im; } cpx;

typedef struct {
  int M;        /* N/2 */
  int logM;
  cpx* twist;   /* exp(i pi j / N), j < M */
  cpx* roots;   /* exp(-2 pi i j / M), j < M/2 */
  int* rev;
} fft_plan;

static fft_plan* plan_create(int N) {
  fft_plan* pl = (fft_plan*)malloc(sizeof(fft_plan));
  pl->M = N / 2;
  pl->logM = ilog2(pl->M);
  pl->twist = (cpx*)malloc(sizeof(cpx) * pl->M);
  pl->roots = (cpx*)malloc(sizeof(cpx) * (pl->M / 2 + 1));
  pl->rev = (int*)malloc(sizeof(int) * pl->M);
  for (int j = 0; j < pl->M; ++j) {
    double ang = M_PI * (double)j / (double)N;
    pl->twist[j].re = cos(ang);
    pl->twist[j].im = sin(ang);
    int r = 0;
    for (int b = 0; b < pl->logM; ++b) if (j & (1 << b)) r |= 1 << (pl->logM - 1 - b);
    pl->rev[j] = r;
  }
  for (int j = 0; j <= pl->M / 2; ++j) {
    double ang = -2.0 * M_PI * (double)j / (double)pl->M;
    pl->roots[j].re = cos(ang);
    pl->roots[j].im = sin(ang);
  }
  return pl;
}

static void plan_destroy(fft_plan* pl) {
  free(pl->twist); free(pl->roots); free(pl->rev); free(pl);
}

/* In-place iterative radix-2 FFT; sign = -1 forward (exp(-2 pi i/M)), +1 inverse (unscaled). */
static void fft_run(const fft_plan* pl, cpx* x, int inverse) {
  const int M = pl->M;
  for (int j = 0; j < M; ++j) {
    int r = pl->rev[j];
    if (r > j) { cpx t = x[j]; x[j] = x[r]; x[r] = t; }
  }
  for (int len = 2; len <= M; len <<= 1) {
    int half = len >> 1, step = M / len;
    for (int s = 0; s < M; s += len) {
      for (int j = 0; j < half; ++j) {
        cpx w = pl->roots[j * step];
        if (inverse) w.im = -w.im;
        cpx u = x[s + j], v = x[s + j + half];
        cpx t = {v.re * w.re - v.im * w.im, v.re * w.im + v.im * w.re};
        x[s + j].re = u.re + t.re; x[s + j].im = u.im + t.im;
        x[s + j + half].re = u.re - t.re; x[s + j + half].im = u.im - t.im;
      }
    }
  }
}

/* Fold a real polynomial (given as signed integers in doubles) and transform. */
static void forward_real(const fft_plan* pl, const double* a, cpx* out) {
  const int M = pl->M;
  for (int j = 0; j < M; ++j) {
    double re = a[j], im = a[j + M];
    cpx w = pl->twist[j];
    out[j].re = re * w.re - im * w.im;
    out[j].im = re * w.im + im * w.re;
  }
  fft_run(pl, out, 0);
}

static inline uint64_t f64_to_torus(double v) {
  double r = rint(v);
  double q = rint(r * 0x1p-64);
  double red = r - q * 0x1p64;
  if (red >= 0x1p63) red -= 0x1p64;
  return (uint64_t)(int64_t)red;
}

/* Inverse transform and add the rounded integer result into out (mod 2^64). */
static void backward_add(const fft_plan* pl, cpx* x, uint64_t* out) {
  const int M = pl->M;
  fft_run(pl, x, 1);
  const double inv = 1.0 / (double)M;
  for (int j = 0; j < M; ++j) {
    cpx w = pl->twist[j];
    double re = (x[j].re * w.re + x[j].im * w.im) * inv;
    double im = (x[j].im * w.re - x[j].re * w.im) * inv;
    out[j] += f64_to_torus(re);
    out[j + M] += f64_to_torus(im);
  }
}

size_t orc_fourier_bsk_doubles(const orc_params* p) {
  return (size_t)p->n * (p->k + 1) * p->pbs_level * (p->k + 1) * p->N; /* M complex = N dbl */
}

void orc_bsk_to_fourier(const orc_params* p, const uint64_t* bsk, double* fbsk) {
  const int N = p->N, polys = p->n * (p->k + 1) * p->pbs_level * (p->k + 1);
  fft_plan* pl = plan_create(N);
#pragma omp parallel
  {
    double* tmp = (double*)malloc(sizeof(double) * N);
#pragma omp for schedule(static)
    for (int q = 0; q < polys; ++q) {
      for (int t = 0; t < N; ++t) tmp[t] = (double)(int64_t)bsk[(size_t)q * N + t];
      forward_real(pl, tmp, (cpx*)(fbsk + (size_t)q * N));
    }
    free(tmp);
  }
  plan_destroy(pl);
}

static void blind_rotate_fft(const orc_params* p, const fft_plan* pl, const double* fbsk,
                             const uint64_t* ct_small, const uint64_t* tv, uint64_t* glwe) {
  const int N = p->N, M = N / 2, k = p->k, l = p->pbs_level, rows = (k + 1) * l, n = p->n;
  const int lg = ilog2(2 * N);
  int bt = modswitch(ct_small[n], lg);
  for (int c = 0; c < k; ++c) memset(glwe + (size_t)c * N, 0, sizeof(uint64_t) * N);
  rotate(N, tv, (2 * N - bt) % (2 * N), glwe + (size_t)k * N);
  uint64_t* rot = (uint64_t*)malloc(sizeof(uint64_t) * N);
  double* dig = (double*)malloc(sizeof(double) * rows * N);
  cpx* dhat = (cpx*)malloc(sizeof(cpx) * rows * M);
  cpx* acc = (cpx*)malloc(sizeof(cpx) * M);
  int64_t dd[64];
  for (int i = 0; i < n; ++i) {
    int ai = modswitch(ct_small[i], lg);
    if (ai == 0) continue;
    for (int c = 0; c <= k; ++c) {
      rotate(N, glwe + (size_t)c * N, ai, rot);
      for (int t = 0; t < N; ++t) {
        decompose(rot[t] - glwe[(size_t)c * N + t], p->pbs_base_log, l, dd);
        for (int j = 0; j < l; ++j) dig[((size_t)c * l + j) * N + t] = (double)dd[j];
      }
    }
    for (int r = 0; r < rows; ++r) forward_real(pl, dig + (size_t)r * N, dhat + (size_t)r * M);
    const cpx* ggsw = (const cpx*)(fbsk + (size_t)i * rows * (k + 1) * N);
    for (int c = 0; c <= k; ++c) {
      for (int t = 0; t < M; ++t) { acc[t].re = 0; acc[t].im = 0; }
      for (int r = 0; r < rows; ++r) {
        const cpx* g = ggsw + ((size_t)r * (k + 1) + c) * M;
        const cpx* d = dhat + (size_t)r * M;
        for (int t = 0; t < M; ++t) {
          acc[t].re += d[t].re * g[t].re - d[t].im * g[t].im;
          acc[t].im += d[t].re * g[t].im + d[t].im * g[t].re;
        }
      }
      backward_add(pl, acc, glwe + (size_t)c * N);
    }
  }
  free(rot); free(dig); free(dhat); free(acc);
}

void orc_pbs_fft(const orc_params* p, const double* fbsk, const uint64_t* ksk,
                 const uint64_t* tv, const uint64_t* in, uint64_t* out, int count, int threads) {
  const int big = p->k * p->N;
  fft_plan* pl = plan_create(p->N);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel
  {
    uint64_t* small = (uint64_t*)malloc(sizeof(uint64_t) * (p->n + 1));
    uint64_t* glwe = (uint64_t*)malloc(sizeof(uint64_t) * (p->k + 1) * p->N);
#pragma omp for schedule(dynamic)
    for (int c = 0; c < count; ++c) {
      orc_keyswitch(p, ksk, in + (size_t)c * (big + 1), small);
      blind_rotate_fft(p, pl, fbsk, small, tv, glwe);
      orc_sample_extract(p, glwe, out + (size_t)c * (big + 1));
    }
    free(small);
    free(glwe);
  }
  plan_destroy(pl);
}

/* ------------------------------------------------------------------------------------------ */
/* Contraction                                                                                 */
/* ------------------------------------------------------------------------------------------ */
void orc_contract(const int64_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                  const uint64_t* X, uint64_t* Y, int batch, int lwe_len, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < batch; ++b) {
    for (int j = 0; j < M; ++j) {
      uint64_t* y = Y + ((size_t)b * M + j) * lwe_len;
      for (int c = 0; c < lwe_len; ++c) y[c] = 0;
      for (int i = 0; i < K; ++i) {
        uint64_t w = (uint64_t)W[(size_t)j * K + i];
        if (!w) continue;
        const uint64_t* x = X + ((size_t)b * K + i) * lwe_len;
        for (int c = 0; c < lwe_len; ++c) y[c] += w * x[c];
      }
      if (bias) y[lwe_len - 1] += (uint64_t)bias[j] * delta;
    }
  }
}
