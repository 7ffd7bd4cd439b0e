// fft1024.cuh -- warp-level negacyclic FFT for polynomials of size N = 2048.
//
// A real polynomial a(X) mod X^N + 1 is folded into M = N/2 complex points
//   y_j = a_j + i a_{j+M},   z_j = y_j * zeta^j,   zeta = exp(i pi / N),
// whose M-point DFT evaluates a(X) at the M roots zeta^(1-4t) of X^N + 1 (those with
// X^(N/2) = i); the conjugate roots follow from a being real.  Products of such transforms are
// negacyclic products.  This is the same "folding" evaluation tfhe-rs performs with its f64
// FFT (tfhe-fft 0.10.1), restated for one warp:
//
//   M = 1024 = 32 x 32 (four-step).  Lane l holds y_{l + 32 m} in register m.
//   forward : twist by zeta^{32 m} (per register) -> in-register DFT32 over m (DIF, output
//             bit-reversed) -> twiddle zeta^l W^{l k2} -> shared-memory transpose ->
//             in-register DFT32 (DIF).  Result: lane l, register r holds
//             Z[32 bitrev(r) + bitrev(l)]  (the "permuted spectrum" order).
//   inverse : exactly the mirror (DIT stages with conjugate twiddles), taking the permuted
//             spectrum back to y'_{l + 32 n} in lane l, register n, scaled by 1/M.
//
// No bit reversal is ever materialised: pointwise products happen in the permuted order, and
// the Fourier bootstrapping key is produced by the same forward routine.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "fft_consts.cuh"

namespace pnb {

constexpr int FFT_R = 32;       // registers (complex) per lane
constexpr int FFT_M = 1024;     // complex points per polynomial
constexpr int FFT_N = 2048;     // polynomial size

// Twiddle tables for one device (all in device global memory).
struct FftTables {
  double2* wf;   // [r*32 + l] = zeta^l * W^{l * bitrev(r)}         (forward, between steps)
  double2* wi;   // [n*32 + l] = zeta^{-n} * W^{-n * bitrev(l)}       (inverse, between steps)
  double2* twf;  // [m] = zeta^{32 m}                                 (forward pre-twist)
  double2* twi;  // [n] = zeta^{-32 n} / M                            (inverse post-twist)
};

// Read-only load the compiler may not hoist out of the blind-rotation loop: the twiddles are
// loop-invariant, and keeping all of them in registers across iterations would spill.
__device__ __forceinline__ double2 ld_tw(const double2* p) {
  double2 v;
  asm volatile("ld.global.nc.v2.f64 {%0, %1}, [%2];" : "=d"(v.x), "=d"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
  return make_double2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ double2 cmul_conj(double2 a, double c, double s) {
  // a * (c - i s)
  return make_double2(fma(a.x, c, a.y * s), fma(a.y, c, -a.x * s));
}
__device__ __forceinline__ double2 cmul_cs(double2 a, double c, double s) {
  // a * (c + i s)
  return make_double2(fma(a.x, c, -a.y * s), fma(a.x, s, a.y * c));
}

// One radix-2 stage of span LEN over the 32 registers.  Templated so that every register
// index is a compile-time constant (a runtime stage length would demote x[] to local memory).
template <int LEN>
__device__ __forceinline__ void dif_stage(double2 (&x)[FFT_R]) {
  constexpr int HALF = LEN / 2;
#pragma unroll
  for (int s = 0; s < 32; s += LEN) {
#pragma unroll
    for (int j = 0; j < HALF; ++j) {
      const double2 u = x[s + j], v = x[s + j + HALF];
      x[s + j] = make_double2(u.x + v.x, u.y + v.y);
      const double2 d = make_double2(u.x - v.x, u.y - v.y);
      const int k = j * (32 / LEN);  // W_LEN^j = W32^k
      if (k == 0) {
        x[s + j + HALF] = d;
      } else if (k == 8) {  // -i
        x[s + j + HALF] = make_double2(d.y, -d.x);
      } else {
        double c, sn;
        w32(k, c, sn);
        x[s + j + HALF] = cmul_cs(d, c, sn);
      }
    }
  }
}

template <int LEN>
__device__ __forceinline__ void dit_stage_inv(double2 (&x)[FFT_R]) {
  constexpr int HALF = LEN / 2;
#pragma unroll
  for (int s = 0; s < 32; s += LEN) {
#pragma unroll
    for (int j = 0; j < HALF; ++j) {
      const int k = j * (32 / LEN);
      const double2 u = x[s + j], v = x[s + j + HALF];
      double2 t;
      if (k == 0) {
        t = v;
      } else if (k == 8) {  // conj(-i) = +i
        t = make_double2(-v.y, v.x);
      } else {
        double c, sn;
        w32(k, c, sn);
        t = cmul_conj(v, c, sn);
      }
      x[s + j] = make_double2(u.x + t.x, u.y + t.y);
      x[s + j + HALF] = make_double2(u.x - t.x, u.y - t.y);
    }
  }
}

// Forward DFT32, decimation in frequency: natural input, bit-reversed output.
__device__ __forceinline__ void dft32_dif(double2 (&x)[FFT_R]) {
  dif_stage<32>(x);
  dif_stage<16>(x);
  dif_stage<8>(x);
  dif_stage<4>(x);
  dif_stage<2>(x);
}

// Inverse DFT32 (exponent +), decimation in time: bit-reversed input, natural output. Unscaled.
__device__ __forceinline__ void idft32_dit(double2 (&x)[FFT_R]) {
  dit_stage_inv<2>(x);
  dit_stage_inv<4>(x);
  dit_stage_inv<8>(x);
  dit_stage_inv<16>(x);
  dit_stage_inv<32>(x);
}

// Swizzled 32x32 transpose through a per-warp shared buffer of 1024 double2.
// Writes element (row = register index, col = lane) and reads back (row = lane, col = register).
__device__ __forceinline__ void warp_transpose(double2 (&x)[FFT_R], double2* buf, int lane) {
#pragma unroll
  for (int r = 0; r < 32; ++r) buf[r * 32 + ((lane + r) & 31)] = x[r];
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q] = buf[lane * 32 + ((q + lane) & 31)];
  __syncwarp();
}

// The same transpose through an 8 KB buffer of 1024 doubles: real parts, then imaginary parts.
__device__ __forceinline__ void warp_transpose_half(double2 (&x)[FFT_R], double* buf, int lane) {
#pragma unroll
  for (int r = 0; r < 32; ++r) buf[r * 32 + ((lane + r) & 31)] = x[r].x;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q].x = buf[lane * 32 + ((q + lane) & 31)];
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 32; ++r) buf[r * 32 + ((lane + r) & 31)] = x[r].y;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 32; ++q) x[q].y = buf[lane * 32 + ((q + lane) & 31)];
  __syncwarp();
}

// Forward / inverse FFT through the 8 KB half buffer.  The forward twiddles come from shared
// memory (`wf_s`, `twf_s`); the inverse ones from the cached global table and `twi_s`.
__device__ __forceinline__ void fft_forward_h(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wf_s, const double2* twf_s) {
#pragma unroll
  for (int m = 0; m < 32; ++m) x[m] = cmul(x[m], twf_s[m]);
  dft32_dif(x);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], wf_s[r * 32 + lane]);
  warp_transpose_half(x, buf, lane);
  dft32_dif(x);
}

__device__ __forceinline__ void fft_inverse_h(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wi_g, const double2* twi_s) {
  idft32_dit(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], __ldg(&wi_g[n * 32 + lane]));
  warp_transpose_half(x, buf, lane);
  idft32_dit(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], twi_s[n]);
}

// Forward twiddle table held once in shared memory for both directions.  Element (a, b) of the
// 32x32 table lives at a*32 + ((a+b) & 31): the forward FFT reads row r across the lanes and the
// inverse reads the transpose (its twiddle (n, lane) is the conjugate of forward element
// (lane, n)); with this swizzle both patterns are bank-conflict free.
__device__ __forceinline__ int tw_swz(int a, int b) { return a * 32 + ((a + b) & 31); }

__device__ __forceinline__ void fft_forward_s(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wf_sw, const double2* twf_s) {
#pragma unroll
  for (int m = 0; m < 32; ++m) x[m] = cmul(x[m], twf_s[m]);
  dft32_dif(x);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], wf_sw[tw_swz(r, lane)]);
  warp_transpose_half(x, buf, lane);
  dft32_dif(x);
}

__device__ __forceinline__ void fft_inverse_s(double2 (&x)[FFT_R], double* buf, int lane,
                                              const double2* wf_sw, const double2* twi_s) {
  idft32_dit(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) {
    const double2 w = wf_sw[tw_swz(lane, n)];  // inverse twiddle = conj(w)
    x[n] = make_double2(fma(x[n].x, w.x, x[n].y * w.y), fma(x[n].x, -w.y, x[n].y * w.x));
  }
  warp_transpose_half(x, buf, lane);
  idft32_dit(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], twi_s[n]);
}

// Forward negacyclic FFT of one folded polynomial (see header comment).
__device__ __forceinline__ void fft_forward(double2 (&x)[FFT_R], double2* buf, int lane,
                                            const FftTables& tb) {
#pragma unroll
  for (int m = 0; m < 32; ++m) x[m] = cmul(x[m], ld_tw(&tb.twf[m]));
  dft32_dif(x);
#pragma unroll
  for (int r = 0; r < 32; ++r) x[r] = cmul(x[r], ld_tw(&tb.wf[r * 32 + lane]));
  warp_transpose(x, buf, lane);
  dft32_dif(x);
}

// Inverse negacyclic FFT back to folded coefficients scaled by 1/M.
__device__ __forceinline__ void fft_inverse(double2 (&x)[FFT_R], double2* buf, int lane,
                                            const FftTables& tb) {
  idft32_dit(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], ld_tw(&tb.wi[n * 32 + lane]));
  warp_transpose(x, buf, lane);
  idft32_dit(x);
#pragma unroll
  for (int n = 0; n < 32; ++n) x[n] = cmul(x[n], ld_tw(&tb.twi[n]));
}

// Host: build (once per device) and fetch the tables of the current device.
int fft_tables_get(FftTables* out);

}  // namespace pnb
