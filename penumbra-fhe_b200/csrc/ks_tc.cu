// ks_tc.cu -- keyswitch on the tensor cores.
//
// The LWE keyswitch of tfhe's KS_PBS order (inside apply_lookup_table, reference call sites
// runtime/src/ops/activation.rs:115 and runtime/src/ops/requant.rs:232) computes, for each
// ciphertext c and output column t,
//     out[c][t] = (t == n ? b_c : 0) - sum_{i < kN, j < L} d[c][i][j] * KSK[i][j][t]   (mod 2^64)
// with signed base-2^ks_base_log digits d in [-B/2, B/2).  As a matrix product this is
//     out = body - D * KSK,   D: [count][kN*L] int8,   KSK: [kN*L][n+1] u64.
// Splitting every u64 KSK word into its 8 little-endian bytes turns KSK into a u8 matrix
// [kN*L][8(n+1)] that is *already laid out* N-contiguous in memory, so tcgen05.mma kind::i8
// reads it as an MN-major B operand without any repacking:
//     C[c][8t + b] = sum_r D[c][r] * byte_b(KSK[r][t])      (exact in s32: |C| < 4*255*10240)
//     out[c][t]    = body - sum_b C[c][8t + b] << 8b        (mod 2^64)
// Tiles: 128 ciphertexts x 256 key bytes (32 output words) per CTA, K staged 128 at a time
// through a 4-deep TMA pipeline, accumulators in TMEM (256 columns).
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "pnb_internal.cuh"
#include "pnb_keys.h"
#include "tc_primitives.cuh"

namespace pnb {

// Device-side status word: non-zero when a bounded wait of a tensor-core kernel ran out.
__device__ int g_tc_status;

int tc_status_read_and_clear(int* out) {
  int v = 0;
  PNB_CUDA(cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int)));
  const int zero = 0;
  PNB_CUDA(cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int)));
  *out = v;
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// Host: TMA descriptors through the driver entry point (no link-time libcuda dependency).
// ------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D u8 tensor [outer][inner] with a row pitch, tiles of box_inner x box_outer, 128B swizzle.
int make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return PNB_ERR_CUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu pitch=%llu", (int)r,
              (unsigned long long)inner, (unsigned long long)outer,
              (unsigned long long)pitch_bytes);
    return PNB_ERR_CUDA;
  }
  return PNB_OK;
}

// ------------------------------------------------------------------------------------------
// Digits: D[c][i*L + j] = signed digit j (most significant first) of in[c][i].
// ------------------------------------------------------------------------------------------
__global__ void ks_digits_kernel(const uint64_t* __restrict__ in, int count, int big, int ld,
                                 int base_log, int level, int8_t* __restrict__ D) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)count * big) return;
  const size_t c = idx / big;
  const int i = (int)(idx % big);
  const uint64_t a = in[c * ld + i];
  const int total = base_log * level;
  uint64_t st = (a >> (64 - total)) + ((a >> (63 - total)) & 1u);
  const uint64_t mask = (1ull << base_log) - 1, half = 1ull << (base_log - 1);
  int8_t* d = D + c * ((size_t)big * level) + (size_t)i * level;
  for (int j = level - 1; j >= 0; --j) {
    const uint64_t v = st & mask;
    st >>= base_log;
    const bool neg = v >= half;
    d[j] = (int8_t)(neg ? (int64_t)v - (int64_t)(1ull << base_log) : (int64_t)v);
    st += neg ? 1u : 0u;
  }
}

// ------------------------------------------------------------------------------------------
// GEMM + limb recombination.
// ------------------------------------------------------------------------------------------
constexpr int KS_BM = 128;                 // ciphertexts per tile
constexpr int KS_BN = 256;                 // key bytes per tile (32 output words)
constexpr int KS_BK = 128;                 // digits per stage
constexpr int KS_STAGES = 4;
constexpr int KS_A_BYTES = KS_BM * KS_BK;  // 16 KB
constexpr int KS_B_BYTES = KS_BK * KS_BN;  // 32 KB (two 128-byte-wide TMA boxes)
constexpr int KS_STAGE_BYTES = KS_A_BYTES + KS_B_BYTES;
constexpr int KS_SMEM = KS_STAGES * KS_STAGE_BYTES + 1024 + 256;
constexpr uint32_t KS_IDESC = tc::idesc_i8(KS_BM, KS_BN, /*a_signed=*/true, /*b_signed=*/false,
                                           /*a_mn=*/false, /*b_mn=*/true);
constexpr uint32_t KS_WAIT_LIMIT = 1u << 24;

__global__ void __launch_bounds__(192, 1) ks_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB,
                                                         const uint64_t* __restrict__ in,
                                                         uint64_t* __restrict__ out, int count,
                                                         int n, int big, int ld, int k_blocks) {
  extern __shared__ unsigned char ks_raw[];
  const uint32_t raw = tc::smem_u32(ks_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bar_base = base + KS_STAGES * KS_STAGE_BYTES;
  auto full = [&](int s) { return bar_base + 8u * s; };
  auto empty = [&](int s) { return bar_base + 8u * (KS_STAGES + s); };
  const uint32_t accum = bar_base + 8u * (2 * KS_STAGES);
  const uint32_t holder = bar_base + 8u * (2 * KS_STAGES + 1);
  unsigned char* holder_ptr = ks_raw + (holder - raw);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * KS_BM;
  const int nb0 = blockIdx.x * KS_BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < KS_STAGES; ++s) {
      tc::mbar_init(full(s), 1);
      tc::mbar_init(empty(s), 1);
    }
    tc::mbar_init(accum, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 1) tc::tmem_alloc(holder, 256);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(holder_ptr);

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int issued = 0;
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int s = kb % KS_STAGES;
        const uint32_t ph = (uint32_t)(kb / KS_STAGES) & 1u;
        if (kb >= KS_STAGES && !tc::mbar_wait(empty(s), ph ^ 1u, KS_WAIT_LIMIT)) {
          atomicExch(&g_tc_status, 1);
          break;
        }
        const uint32_t a_s = base + s * KS_STAGE_BYTES, b_s = a_s + KS_A_BYTES;
        tc::mbar_expect_tx(full(s), KS_STAGE_BYTES);
        tc::tma_load_2d(a_s, &tmA, kb * KS_BK, m0, full(s));
        tc::tma_load_2d(b_s, &tmB, nb0, kb * KS_BK, full(s));
        tc::tma_load_2d(b_s + KS_BK * 128, &tmB, nb0 + 128, kb * KS_BK, full(s));
        issued = kb + 1;
      }
      // No copy may still be landing when the block exits: observe (bounded) the completion
      // of the last use of every stage -- immediate unless a wait above ran out.
      for (int kb = issued > KS_STAGES ? issued - KS_STAGES : 0; kb < issued; ++kb)
        (void)tc::mbar_wait(full(kb % KS_STAGES), (uint32_t)(kb / KS_STAGES) & 1u, KS_WAIT_LIMIT);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int s = kb % KS_STAGES;
        const uint32_t ph = (uint32_t)(kb / KS_STAGES) & 1u;
        if (!tc::mbar_wait(full(s), ph, KS_WAIT_LIMIT)) {
          atomicExch(&g_tc_status, 2);
          break;
        }
        tc::tc_fence_after();
        const uint32_t a_s = base + s * KS_STAGE_BYTES, b_s = a_s + KS_A_BYTES;
#pragma unroll
        for (int k = 0; k < KS_BK / 32; ++k) {
          // A: K-major, advance 32 bytes along K inside the 128-byte swizzled row.
          const uint64_t ad = tc::smem_desc_sw128(a_s + 32u * k, 16u, 1024u);
          // B: MN-major, 32 K-rows = 4 swizzle atoms of 1024 bytes; MN blocks 16 KB apart.
          const uint64_t bd = tc::smem_desc_sw128(b_s + 4096u * k, (uint32_t)(KS_BK * 128), 1024u);
          tc::mma_i8(tmem, ad, bd, KS_IDESC, (kb | k) != 0 ? 1u : 0u);
        }
        tc::mma_commit(empty(s));
      }
      tc::mma_commit(accum);
    }
  } else {  // epilogue: warps 2..5 cover TMEM lane quarters 2, 3, 0, 1
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    if (tc::mbar_wait(accum, 0, KS_WAIT_LIMIT)) {
      tc::tc_fence_after();
      const int col0 = nb0 / 8;
      const uint64_t body = (row < count) ? in[(size_t)row * ld + big] : 0;
#pragma unroll 1
      for (int chunk = 0; chunk < KS_BN / 32; ++chunk) {
        uint32_t r[32];
        tc::tmem_ld_32x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(chunk * 32), r);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint64_t v = 0;
#pragma unroll
          for (int b = 0; b < 8; ++b) v += (uint64_t)(int64_t)(int32_t)r[u * 8 + b] << (8 * b);
          const int col = col0 + chunk * 4 + u;
          if (row < count && col <= n) out[(size_t)row * (n + 1) + col] = (col == n ? body : 0) - v;
        }
      }
    } else {
      atomicExch(&g_tc_status, 3);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

size_t ks_tc_workspace_bytes(const pnb_params& p, int count) {
  const size_t d = (size_t)count * p.k * p.N * p.ks_level;
  return (d + 255) & ~(size_t)255;
}

// in: [count][in_ld] big-key ciphertexts (kN+1 words used; in_ld 0 = kN+1); out: [count][n+1];
// digits: scratch of ks_tc_workspace_bytes.
int keyswitch_tc(const pnb_keys* K, const uint64_t* in, uint64_t* out, int count, void* digits,
                 cudaStream_t st, int in_ld) {
  const pnb_params& p = K->p;
  const int big = p.k * p.N;
  const int ld = in_ld > 0 ? in_ld : big + 1;
  if (ld < big + 1) {
    set_error("keyswitch: row pitch %d is shorter than a %d-word ciphertext", ld, big + 1);
    return PNB_ERR_INVALID;
  }
  const int kdim = big * p.ks_level;
  if (kdim % KS_BK != 0 || p.ks_base_log > 7 || p.ks_base_log < 1 ||
      p.ks_base_log * p.ks_level >= 64) {
    set_error("keyswitch: unsupported shape kN*ks_level=%d ks_base_log=%d", kdim, p.ks_base_log);
    return PNB_ERR_UNSUPPORTED;
  }
  if (count <= 0) return PNB_OK;
  if ((uintptr_t)digits % 16 != 0) {
    set_error("keyswitch: digit scratch must be 16-byte aligned");
    return PNB_ERR_INVALID;
  }
  int8_t* D = static_cast<int8_t*>(digits);
  const size_t tot = (size_t)count * big;
  ks_digits_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(in, count, big, ld,
                                                                 p.ks_base_log, p.ks_level, D);
  PNB_CHECK_LAUNCH("ks_digits_kernel");
  CUtensorMap tmA, tmB;
  int rc = make_tmap_u8_2d(&tmA, D, (uint64_t)kdim, (uint64_t)count, (uint64_t)kdim, KS_BK,
                           KS_BM);
  if (rc) return rc;
  const uint64_t key_bytes = (uint64_t)K->ksk_row * 8;
  rc = make_tmap_u8_2d(&tmB, K->ksk, key_bytes, (uint64_t)kdim, key_bytes, 128, KS_BK);
  if (rc) return rc;
  static bool attr_done[64];
  int dev = 0;
  PNB_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    PNB_CUDA(cudaFuncSetAttribute(ks_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  KS_SMEM));
    attr_done[dev] = true;
  }
  const int n_tiles = (int)((8 * (uint64_t)(p.n + 1) + KS_BN - 1) / KS_BN);
  const int m_tiles = (count + KS_BM - 1) / KS_BM;
  if (m_tiles > 65535) {
    set_error("keyswitch: %d ciphertexts exceed one launch (max %d)", count, 65535 * KS_BM);
    return PNB_ERR_INVALID;
  }
  dim3 grid(n_tiles, m_tiles);
  ks_gemm_kernel<<<grid, 192, KS_SMEM, st>>>(tmA, tmB, in, out, count, p.n, big, ld,
                                             kdim / KS_BK);
  PNB_CHECK_LAUNCH("ks_gemm_kernel");
  return PNB_OK;
}

}  // namespace pnb
