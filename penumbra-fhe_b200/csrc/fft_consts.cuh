// Generated constants: exp(-2 pi i k / 32) for k = 0..15 as (cos, sin) pairs, hex floats.
#pragma once
namespace pnb {
__device__ __forceinline__ void w32(int k, double& c, double& s) {
  switch (k) {
    case 0: c = 0x1.0000000000000p+0; s = 0x0.0p+0; break;
    case 1: c = 0x1.f6297cff75cb0p-1; s = -0x1.8f8b83c69a60ap-3; break;
    case 2: c = 0x1.d906bcf328d46p-1; s = -0x1.87de2a6aea963p-2; break;
    case 3: c = 0x1.a9b66290ea1a3p-1; s = -0x1.1c73b39ae68c8p-1; break;
    case 4: c = 0x1.6a09e667f3bcdp-1; s = -0x1.6a09e667f3bccp-1; break;
    case 5: c = 0x1.1c73b39ae68c9p-1; s = -0x1.a9b66290ea1a3p-1; break;
    case 6: c = 0x1.87de2a6aea964p-2; s = -0x1.d906bcf328d46p-1; break;
    case 7: c = 0x1.8f8b83c69a60dp-3; s = -0x1.f6297cff75cb0p-1; break;
    case 8: c = 0x0.0p+0; s = -0x1.0000000000000p+0; break;
    case 9: c = -0x1.8f8b83c69a608p-3; s = -0x1.f6297cff75cb0p-1; break;
    case 10: c = -0x1.87de2a6aea962p-2; s = -0x1.d906bcf328d46p-1; break;
    case 11: c = -0x1.1c73b39ae68c6p-1; s = -0x1.a9b66290ea1a5p-1; break;
    case 12: c = -0x1.6a09e667f3bccp-1; s = -0x1.6a09e667f3bcdp-1; break;
    case 13: c = -0x1.a9b66290ea1a4p-1; s = -0x1.1c73b39ae68c8p-1; break;
    case 14: c = -0x1.d906bcf328d46p-1; s = -0x1.87de2a6aea965p-2; break;
    case 15: c = -0x1.f6297cff75cb0p-1; s = -0x1.8f8b83c69a617p-3; break;
    default: c = 1.0; s = 0.0; break;
  }
}
}  // namespace pnb
