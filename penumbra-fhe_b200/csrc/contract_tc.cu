// contract_tc.cu -- ciphertext x cleartext-weight contraction on the tensor cores.
//
// Replaces the scalar_mul_parallelized / add_parallelized / scalar_add_parallelized loops of
// Linear::eval (runtime/src/ops/linear.rs:52-75), Conv2d::eval (runtime/src/ops/conv2d.rs:91-139)
// and the window sums of Pool::eval (runtime/src/ops/pool.rs:110-118).  All three are
//     Y[g][j][c] = sum_k W[j][k] * X[idx[g][k]][c]   (+ bias[j] * delta on the body c = L-1)
// over LWE ciphertexts of L words mod 2^64: a Linear layer is idx[g][k] = g*K + k, a
// convolution is an implicit im2col (idx = input ciphertext under tap k of output position g,
// -1 for zero padding), an average pool is W = 1 over the window.
//
// Each u64 word is 8 little-endian bytes, so for one group g the operand X[idx[g][:]][:] is a
// u8 matrix [K][8L] that is N-contiguous: tcgen05.mma kind::i8 consumes it as an MN-major B
// operand (A = W, s8, K-major) and the epilogue recombines the 8 byte-limb accumulators:
//     Y = sum_b C[.][8c + b] << 8b   (mod 2^64),  |C| <= 128 * 255 * K < 2^31 for K < 65794.
//
// Ciphertext rows hold L = kN+1 words at a row pitch ld >= L.  How the B tiles reach shared
// memory (in the SWIZZLE_128B layout the MMA reads) depends on the pitch:
//   dense rows at an even pitch (16-byte aligned rows, the layout the graph evaluator keeps):
//     two TMA tiles of 128 rows x 128 bytes per stage, issued by one thread;
//   gathered rows (convolutions, pools) at an even pitch: 16-byte cp.async.cg copies by 8 warps
//     (L2 only: in-flight copies take no L1 lines);
//   rows at an odd pitch (contiguous [count][kN+1] ciphertexts): 8-byte cp.async.ca copies, the
//     only form that reaches every word, with fewer stages because in-flight 8-byte copies hold
//     L1 lines, and L1 shares the SM's 256 KB with shared memory.
// W (padded on the device to [Mp][Kp]) comes by TMA, one tile per stage.  Persistent CTAs walk
// (group, M tile, N tile) tiles; 1 warp issues MMAs, 4 warps run the epilogue from
// double-buffered TMEM accumulators (2 x 256 columns).
#include <cudaTypedefs.h>

#include <cstdio>

#include "pnb_internal.cuh"
#include "pnb_keys.h"
#include "tc_primitives.cuh"

namespace pnb {

// Status word of the contraction kernel: non-zero when one of its bounded waits ran out.
__device__ int g_ct_status;

int ct_status_read_and_clear(int* out) {
  int v = 0;
  PNB_CUDA(cudaMemcpyFromSymbol(&v, g_ct_status, sizeof(int)));
  const int zero = 0;
  PNB_CUDA(cudaMemcpyToSymbol(g_ct_status, &zero, sizeof(int)));
  *out = v;
  return PNB_OK;
}

int make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer);

constexpr int CT_BM = 128;                   // output rows per tile
constexpr int CT_BN = 256;                   // B bytes per tile = 32 output words
constexpr int CT_BK = 128;                   // K per stage
// B operand modes (see the header comment).
enum : int { CT_GATHER8 = 0, CT_GATHER16 = 1, CT_DENSE_TMA = 2 };
// Three stages for 8-byte gathers: they hold their data in L1 lines while in flight, so every
// kilobyte of shared memory given to a fourth stage is taken from the bytes that can be in
// flight (measured: 4 stages 1.44 ms, 3 stages 1.17 ms for 256 samples of Linear 784 -> 128).
// The other modes keep nothing in L1 and take four.
constexpr int CT_STAGES = 3;
constexpr int CT_STAGES_WIDE = 4;
__host__ __device__ constexpr int ct_stages(int mode) {
  return mode == CT_GATHER8 ? CT_STAGES : CT_STAGES_WIDE;
}
constexpr int CT_A_BYTES = CT_BM * CT_BK;    // 16 KB
constexpr int CT_B_BYTES = CT_BK * CT_BN;    // 32 KB
constexpr int CT_STAGE_BYTES = CT_A_BYTES + CT_B_BYTES;
#ifndef CT_PROD_WARPS
#define CT_PROD_WARPS 8
#endif
constexpr int CT_PW = CT_PROD_WARPS;          // gathering warps 0..CT_PW-1
constexpr int CT_PRODUCERS = 32 * CT_PW;
constexpr int CT_ROWS_PER_WARP = CT_BK / CT_PW;
constexpr int CT_MMA_WARP = CT_PW;
#ifndef CT_EPI_WARP_COUNT
#define CT_EPI_WARP_COUNT 4
#endif
constexpr int CT_EPI_WARPS = CT_EPI_WARP_COUNT;      // 4 or 8: one or two per TMEM lane quarter
constexpr int CT_EPI_WORDS = 32 * 4 / CT_EPI_WARPS;  // output words per epilogue warp (32 / 16)
constexpr int CT_EPI_CPAIRS = CT_EPI_WORDS / 8;      // chunk pairs (2 x 4 words) per warp
constexpr int CT_THREADS = 32 * (CT_PW + 1 + CT_EPI_WARPS);
constexpr int CT_EPI_BYTES = CT_EPI_WARPS * 32 * 8 * 8;  // per warp: 32 rows x 8 words
// 1024-byte alignment slack, the stage ring, 256 bytes of barriers, the epilogue staging
__host__ __device__ constexpr int ct_smem(int mode) {
  return 1024 + ct_stages(mode) * CT_STAGE_BYTES + 256 + CT_EPI_BYTES;
}
constexpr uint32_t CT_IDESC = tc::idesc_i8(CT_BM, CT_BN, /*a_signed=*/true,
                                           /*b_signed=*/false, /*a_mn=*/false, /*b_mn=*/true);
constexpr uint32_t CT_WAIT_LIMIT = 1u << 24;

struct CtArgs {
  const uint64_t* X;       // ciphertexts [*][ldx] (L words used)
  const int32_t* idx;      // [G][K] ciphertext index into X, -1 = zero
  const int64_t* bias;     // [M] or null
  uint64_t* Y;             // [G][M][ldy], or [G/P][M][P][ldy] when P > 0
  uint64_t delta;
  int G, M, K, L;
  int ldx, ldy;            // row pitches of X and Y in words
  int P;                   // output positions per sample (channel-major placement); 0 = off
  int m_tiles, n_tiles, k_blocks;
};

__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}

// Bounded wait that also gives up as soon as another role has flagged an abort.
__device__ __forceinline__ bool ct_wait(uint32_t bar, uint32_t parity, volatile int* abort_s) {
  for (uint32_t it = 0; it < CT_WAIT_LIMIT; it += 1024) {
    if (tc::mbar_wait(bar, parity, 1024)) return true;
    if (*abort_s) return false;
  }
  *abort_s = 1;
  atomicExch(&g_ct_status, 1);
  return false;
}

template <int MODE>
__global__ void __launch_bounds__(CT_THREADS, 1) contract_tc_kernel(
    const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
    CtArgs a) {
  constexpr int STAGES = ct_stages(MODE);
  extern __shared__ unsigned char ct_raw[];
  const uint32_t raw = tc::smem_u32(ct_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  auto stage_at = [&](int s) { return base + (uint32_t)(s * CT_STAGE_BYTES); };
  const uint32_t bars = base + STAGES * CT_STAGE_BYTES;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (STAGES + s); };
  auto acc_full = [&](int b) { return bars + 8u * (2 * STAGES + b); };
  auto acc_empty = [&](int b) { return bars + 8u * (2 * STAGES + 2 + b); };
  const uint32_t holder = bars + 8u * (2 * STAGES + 4);
  volatile int* abort_s = reinterpret_cast<volatile int*>(ct_raw + (holder + 8 - raw));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // TMA stages complete by transaction count alone; gathered stages also need every
      // producer thread's arrival
      tc::mbar_init(full(s), MODE == CT_DENSE_TMA ? 1 : CT_PRODUCERS + 1);
      tc::mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(acc_full(b), 1);
      tc::mbar_init(acc_empty(b), 32 * CT_EPI_WARPS);
    }
    *abort_s = 0;
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmW);
    if (MODE == CT_DENSE_TMA) tc::prefetch_tmap(&tmX);
  }
  if (warp == CT_MMA_WARP) tc::tmem_alloc(holder, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(ct_raw + (holder - raw));

  const int total = a.G * a.m_tiles * a.n_tiles;

  if (MODE == CT_DENSE_TMA && warp < CT_PW) {
    // ---------------- TMA producer: one thread, three tiles per stage -----------------------
    // Group g's K rows are rows g*K .. g*K + K-1 of X; the rows past K in the last stage belong
    // to the next group (or lie past the tensor and read as zeros) and meet zero weights.
    if (warp == 0 && lane == 0) {
      int kb_global = 0;
      for (int t = blockIdx.x; t < total && !*abort_s; t += gridDim.x) {
        const int nt = t % a.n_tiles;
        const int mt = (t / a.n_tiles) % a.m_tiles;
        const int g = t / (a.n_tiles * a.m_tiles);
        bool ok = true;
        for (int kb = 0; kb < a.k_blocks; ++kb, ++kb_global) {
          const int s = kb_global % STAGES;
          const uint32_t use = (uint32_t)(kb_global / STAGES);
          if (use > 0 && !ct_wait(empty(s), (use - 1) & 1u, abort_s)) { ok = false; break; }
          const uint32_t a_s = stage_at(s);
          const uint32_t b_s = a_s + CT_A_BYTES;
          tc::mbar_expect_tx(full(s), CT_STAGE_BYTES);
          tc::tma_load_2d(a_s, &tmW, kb * CT_BK, mt * CT_BM, full(s));
          const int row = g * a.K + kb * CT_BK;
          tc::tma_load_2d(b_s, &tmX, nt * CT_BN, row, full(s));
          tc::tma_load_2d(b_s + CT_BK * 128, &tmX, nt * CT_BN + 128, row, full(s));
        }
        if (!ok) break;
      }
      // no tile may still be landing when the block exits: the last use of each stage
      // completes when its tiles have landed (bounded; immediate unless a wait ran out)
      for (int k = kb_global > STAGES ? kb_global - STAGES : 0; k < kb_global; ++k)
        (void)tc::mbar_wait(full(k % STAGES), (uint32_t)(k / STAGES) & 1u, CT_WAIT_LIMIT);
    }
  } else if (MODE == CT_GATHER16 && warp < CT_PW) {
    // ---------------- 16-byte gather producers: each instruction of a warp copies two rows
    // of 256 bytes (16 lanes per row); warp w fills rows 16w .. 16w + 15 of every stage.
    constexpr int CT_LAG = STAGES - 1;
    constexpr int RPW = CT_BK / CT_PW;  // rows per warp per stage
    int kb_global = 0, released = 0;
    for (int t = blockIdx.x; t < total && !*abort_s; t += gridDim.x) {
      const int nt = t % a.n_tiles;
      const int mt = (t / a.n_tiles) % a.m_tiles;
      const int g = t / (a.n_tiles * a.m_tiles);
      const int c16 = lane & 15;                  // 16-byte chunk of the 256-byte row piece
      const int w0 = nt * 32 + 2 * c16;           // its first word
      const bool col_ok = w0 < a.L;               // (w0 + 1 < ldx: the pitch is even)
      const int box = c16 >> 3, ch = c16 & 7;
      const int32_t* idx_g = a.idx ? a.idx + (size_t)g * a.K : nullptr;
      for (int kb = 0; kb < a.k_blocks; ++kb, ++kb_global) {
        const int s = kb_global % STAGES;
        const uint32_t use = (uint32_t)(kb_global / STAGES);
        if (use > 0 && !ct_wait(empty(s), (use - 1) & 1u, abort_s)) break;
        const uint32_t a_s = stage_at(s);
        const uint32_t b_s = a_s + CT_A_BYTES;
        if (warp == 0 && lane == 0) {  // the W tile of this stage, by TMA
          tc::mbar_expect_tx(full(s), CT_A_BYTES);
          tc::tma_load_2d(a_s, &tmW, kb * CT_BK, mt * CT_BM, full(s));
        }
        // lane i < RPW holds the index of row k = kb*CT_BK + RPW*warp + i
        const int kr = kb * CT_BK + RPW * warp + lane;
        const int my_idx = (lane >= RPW || kr >= a.K) ? -1
                           : idx_g ? __ldg(idx_g + kr) : g * a.K + kr;
#pragma unroll 4
        for (int j = 0; j < RPW / 2; ++j) {
          const int ri = 2 * j + (lane >> 4);
          const int r = RPW * warp + ri;  // row within the stage
          const int x = __shfl_sync(0xffffffffu, my_idx, ri);
          const bool ok = col_ok && x >= 0;
          const uint64_t* src = ok ? a.X + (size_t)x * a.ldx + w0 : a.X;
          const uint32_t dst = b_s + box * (CT_BK * 128) + (r >> 3) * 1024 + (r & 7) * 128 +
                               ((ch ^ (r & 7)) << 4);
          cp_async16(dst, src, ok ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (kb_global + 1 - released > CT_LAG) {
          asm volatile("cp.async.wait_group %0;" ::"n"(CT_LAG) : "memory");
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc::mbar_arrive(full(released % STAGES));
          ++released;
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (; released < kb_global; ++released) tc::mbar_arrive(full(released % STAGES));
    if (warp == 0 && lane == 0) {
      for (int k = kb_global > STAGES ? kb_global - STAGES : 0; k < kb_global; ++k)
        (void)tc::mbar_wait(full(k % STAGES), (uint32_t)(k / STAGES) & 1u, CT_WAIT_LIMIT);
    }
  } else if (warp < CT_PW) {
    // ---------------- gather producers: CT_PW warps x 32 columns, CT_BK/CT_PW rows each -------
    // Copies of up to CT_LAG stages stay in flight; stage kb_global - CT_LAG is released (its
    // mbarrier arrive) once its group has landed.  CT_LAG <= CT_STAGES - 1 keeps the ring live:
    // refilling stage s waits for the MMAs of its previous use, released CT_LAG groups earlier.
    constexpr int CT_LAG = STAGES - 1;
    int kb_global = 0, released = 0;
    for (int t = blockIdx.x; t < total && !*abort_s; t += gridDim.x) {
      const int nt = t % a.n_tiles;
      const int mt = (t / a.n_tiles) % a.m_tiles;
      const int g = t / (a.n_tiles * a.m_tiles);
      const int col = nt * 32 + lane;
      const bool col_ok = col < a.L;
      const int32_t* idx_g = a.idx ? a.idx + (size_t)g * a.K : nullptr;
      for (int kb = 0; kb < a.k_blocks; ++kb, ++kb_global) {
        const int s = kb_global % STAGES;
        const uint32_t use = (uint32_t)(kb_global / STAGES);
        if (use > 0 && !ct_wait(empty(s), (use - 1) & 1u, abort_s)) break;
        const uint32_t a_s = stage_at(s);
        const uint32_t b_s = a_s + CT_A_BYTES;
        if (warp == 0 && lane == 0) {  // the W tile of this stage, by TMA
          tc::mbar_expect_tx(full(s), CT_A_BYTES);
          tc::tma_load_2d(a_s, &tmW, kb * CT_BK, mt * CT_BM, full(s));
        }
        // lane i < CT_ROWS_PER_WARP holds the index of row k = kb*CT_BK + warp + CT_PW*i
        const int kr = kb * CT_BK + warp + CT_PW * lane;
        // dense operand (idx == null): ciphertext g*K + k
        const int my_idx = (kr >= a.K) ? -1 : idx_g ? __ldg(idx_g + kr) : g * a.K + kr;
        const int box = lane >> 4, ch = (lane & 15) >> 1, half = lane & 1;
#pragma unroll 4
        for (int i = 0; i < CT_ROWS_PER_WARP; ++i) {
          const int r = warp + CT_PW * i;  // row within the stage
          const int x = __shfl_sync(0xffffffffu, my_idx, i);
          const bool ok = col_ok && x >= 0;
          const uint64_t* src = ok ? a.X + (size_t)x * a.ldx + col : a.X;
          const uint32_t dst = b_s + box * (CT_BK * 128) + (r >> 3) * 1024 + (r & 7) * 128 +
                               ((ch ^ (r & 7)) << 4) + half * 8;
          cp_async8(dst, src, ok ? 8u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (kb_global + 1 - released > CT_LAG) {
          asm volatile("cp.async.wait_group %0;" ::"n"(CT_LAG) : "memory");
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc::mbar_arrive(full(released % STAGES));
          ++released;
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (; released < kb_global; ++released) tc::mbar_arrive(full(released % STAGES));
    if (warp == 0 && lane == 0) {
      // No W tile may still be landing when the block exits.  Every producer has arrived for
      // every stage it filled (above), so the last use of each stage completes exactly when its
      // W tile has landed: observe that (bounded) -- immediate unless a wait ran out.
      for (int k = kb_global > STAGES ? kb_global - STAGES : 0; k < kb_global; ++k)
        (void)tc::mbar_wait(full(k % STAGES), (uint32_t)(k / STAGES) & 1u, CT_WAIT_LIMIT);
    }
  } else if (warp == CT_MMA_WARP) {
    // ---------------- MMA issue (one elected lane) --------------------------------------------
    if (lane == 0) {
      int kb_global = 0, tt = 0;
      for (int t = blockIdx.x; t < total && !*abort_s; t += gridDim.x, ++tt) {
        const int buf = tt & 1;
        const uint32_t d_tmem = tmem + (uint32_t)(buf * 256);
        if (tt >= 2 && !ct_wait(acc_empty(buf), (uint32_t)((tt >> 1) - 1) & 1u, abort_s)) break;
        tc::tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < a.k_blocks; ++kb, ++kb_global) {
          const int s = kb_global % STAGES;
          const uint32_t use = (uint32_t)(kb_global / STAGES);
          const uint32_t a_s = stage_at(s);
          if (!ct_wait(full(s), use & 1u, abort_s)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t b_s = a_s + CT_A_BYTES;
#pragma unroll
          for (int k = 0; k < CT_BK / 32; ++k) {
            const uint64_t ad = tc::smem_desc_sw128(a_s + 32u * k, 16u, 1024u);
            const uint64_t bd = tc::smem_desc_sw128(b_s + 4096u * k, (uint32_t)(CT_BK * 128),
                                                    1024u);
            tc::mma_i8(d_tmem, ad, bd, CT_IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          tc::mma_commit(empty(s));
        }
        if (!ok) break;
        tc::mma_commit(acc_full(buf));
      }
    }
  } else {
    // ---------------- epilogue: the last CT_EPI_WARPS warps ----------------------------------
    // Warp w reads TMEM lane quarter w % 4 (its 32 output rows) and its share of the tile's 32
    // output words, in chunk pairs of 2 x 32 columns = 8 words of 8 byte-limbs each.  The limbs
    // are recombined into u64 words, staged in shared memory (32 rows x 8 words, XOR-swizzled)
    // and written out as 64-byte row segments, one chunk pair at a time; the TMEM buffer is
    // released as soon as its last chunk pair has been read.
    const int e_w = warp - CT_MMA_WARP - 1;
    const int q = warp & 3, eh = e_w >> 2;
    constexpr int EW = CT_EPI_WORDS;
    uint64_t* stage = reinterpret_cast<uint64_t*>(ct_raw + (bars + 256 - raw)) +
                      (size_t)e_w * 32 * 8;
    int tt = 0;
    for (int t = blockIdx.x; t < total && !*abort_s; t += gridDim.x, ++tt) {
      const int nt = t % a.n_tiles;
      const int mt = (t / a.n_tiles) % a.m_tiles;
      const int g = t / (a.n_tiles * a.m_tiles);
      const int buf = tt & 1;
      if (!ct_wait(acc_full(buf), (uint32_t)(tt >> 1) & 1u, abort_s)) break;
      tc::tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t)(buf * 256) + ((uint32_t)(q * 32) << 16) +
                             (uint32_t)(eh * (EW / 4) * 32);
#pragma unroll 1
      for (int cp = 0; cp < CT_EPI_CPAIRS; ++cp) {
        uint32_t r0[32], r1[32];
        tc::tmem_ld_32x32_nowait(tbase + (uint32_t)(cp * 64), r0);
        tc::tmem_ld_32x32_nowait(tbase + (uint32_t)(cp * 64 + 32), r1);
        tc::tmem_ld_wait();
        if (cp == CT_EPI_CPAIRS - 1) {
          tc::tc_fence_before();
          tc::mbar_arrive(acc_empty(buf));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          uint64_t v = 0;
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            const uint32_t c = u < 4 ? r0[u * 8 + b] : r1[(u - 4) * 8 + b];
            v += (uint64_t)(int64_t)(int32_t)c << (8 * b);
          }
          stage[lane * 8 + (u ^ (lane & 7))] = v;
        }
        __syncwarp();
        // 4 rows per instruction, 8 lanes x 8 bytes = one 64-byte row segment each
        const int w = lane & 7;
        const int col = nt * 32 + eh * EW + cp * 8 + w;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + (lane >> 3);
          const int row = mt * CT_BM + q * 32 + rr;
          uint64_t v = stage[rr * 8 + (w ^ (rr & 7))];
          if (row < a.M && col < a.L) {
            if (col == a.L - 1 && a.bias) v += (uint64_t)a.bias[row] * a.delta;
            const size_t yr = a.P > 0 ? ((size_t)(g / a.P) * a.M + row) * a.P + (g % a.P)
                                      : (size_t)g * a.M + row;
            a.Y[yr * a.ldy + col] = v;
          }
        }
        __syncwarp();
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == CT_MMA_WARP) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// W int8 [M][K] -> zero-padded [Mp][Kp] (Mp, Kp multiples of 128).
__global__ void pad_weights_kernel(const int8_t* __restrict__ W, int M, int K, int8_t* Wp,
                                   int Mp, int Kp) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)Mp * Kp) return;
  const int r = (int)(i / Kp), c = (int)(i % Kp);
  Wp[i] = (r < M && c < K) ? W[(size_t)r * K + c] : (int8_t)0;
}

// idx[g][k] = g*K + k: the dense (Linear) gather.

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

int lwe_contract_gather(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                        const uint64_t* X, const int32_t* idx, int G, uint64_t* Y, int L,
                        cudaStream_t st) {
  return lwe_contract_gather_placed(W, bias, delta, M, K, X, idx, G, Y, L, 0, st);
}

template <int MODE>
static int ct_launch(int grid, const CUtensorMap& tmW, const CUtensorMap& tmX, const CtArgs& a,
                     cudaStream_t st) {
  static bool attr_done[64];
  int dev = 0;
  PNB_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    PNB_CUDA(cudaFuncSetAttribute(contract_tc_kernel<MODE>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, ct_smem(MODE)));
    attr_done[dev] = true;
  }
  contract_tc_kernel<MODE><<<grid, CT_THREADS, ct_smem(MODE), st>>>(tmW, tmX, a);
  PNB_CHECK_LAUNCH("contract_tc_kernel");
  return PNB_OK;
}

int lwe_contract_gather_placed(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                               const uint64_t* X, const int32_t* idx, int G, uint64_t* Y, int L,
                               int P, cudaStream_t st, int ldx, int ldy) {
  if (ldx == 0) ldx = L;
  if (ldy == 0) ldy = L;
  if (ldx < L || ldy < L) {
    set_error("contract: row pitches %d / %d are shorter than the %d-word rows", ldx, ldy, L);
    return PNB_ERR_INVALID;
  }
  // 16-byte copies need rows that start 16-byte aligned: an even pitch and an aligned base
  const bool even = (ldx % 2) == 0 && ((uintptr_t)X % 16) == 0;
  const int mode = !even ? CT_GATHER8 : (idx == nullptr ? CT_DENSE_TMA : CT_GATHER16);
  if (P < 0 || (P > 0 && G % P != 0)) {
    set_error("contract: %d groups are not a whole number of samples of %d positions", G, P);
    return PNB_ERR_INVALID;
  }
  if (M <= 0 || K <= 0 || G < 0 || L <= 0 || K > 65536) {
    set_error("contract: bad shape M=%d K=%d groups=%d L=%d (K <= 65536)", M, K, G, L);
    return PNB_ERR_INVALID;
  }
  if (G == 0) return PNB_OK;
  const int Mp = (M + CT_BM - 1) / CT_BM * CT_BM, Kp = (K + CT_BK - 1) / CT_BK * CT_BK;
  int8_t* Wp = nullptr;
  PNB_CUDA(cudaMallocAsync((void**)&Wp, (size_t)Mp * Kp, st));
  const size_t nw = (size_t)Mp * Kp;
  pad_weights_kernel<<<(unsigned)((nw + 255) / 256), 256, 0, st>>>(W, M, K, Wp, Mp, Kp);
  int rc = PNB_OK;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = cuda_status(e, "pad_weights_kernel");
  CUtensorMap tmW;
  if (rc == PNB_OK) rc = make_tmap_u8_2d(&tmW, Wp, (uint64_t)Kp, (uint64_t)Mp, (uint64_t)Kp,
                                         CT_BK, CT_BM);
  // the dense operand as a 2D byte tensor [rows][8 ldx] for the TMA mode
  CUtensorMap tmX{};
  if (rc == PNB_OK && mode == CT_DENSE_TMA)
    rc = make_tmap_u8_2d(&tmX, X, (uint64_t)ldx * 8, (uint64_t)G * K, (uint64_t)ldx * 8, 128,
                         CT_BK);
  if (rc == PNB_OK) {
    CtArgs args;
    args.X = X; args.idx = idx; args.bias = bias; args.Y = Y; args.delta = delta;
    args.G = G; args.M = M; args.K = K; args.L = L; args.P = P;
    args.ldx = ldx; args.ldy = ldy;
    args.m_tiles = Mp / CT_BM;
    args.n_tiles = (8 * L + CT_BN - 1) / CT_BN;
    args.k_blocks = Kp / CT_BK;
    const long long tiles = (long long)G * args.m_tiles * args.n_tiles;
    if (tiles > 0x7fffffffLL) {
      set_error("contract: %lld tiles exceed one launch", tiles);
      rc = PNB_ERR_INVALID;
    } else {
      const int grid = (int)std::min<long long>(tiles, (long long)sm_count());
      rc = mode == CT_DENSE_TMA ? ct_launch<CT_DENSE_TMA>(grid, tmW, tmX, args, st)
         : mode == CT_GATHER16  ? ct_launch<CT_GATHER16>(grid, tmW, tmX, args, st)
                                : ct_launch<CT_GATHER8>(grid, tmW, tmX, args, st);
    }
  }
  e = cudaFreeAsync(Wp, st);
  if (rc == PNB_OK && e != cudaSuccess) rc = cuda_status(e, "cudaFreeAsync(padded weights)");
  return rc;
}

int lwe_contract_tc(const int8_t* W, const int64_t* bias, uint64_t delta, int M, int K,
                    const uint64_t* X, uint64_t* Y, int batch, int L, cudaStream_t st, int ldx,
                    int ldy) {
  if (batch <= 0) return batch == 0 ? PNB_OK : PNB_ERR_INVALID;
  if ((long long)batch * K > 0x7fffffffLL) {
    set_error("contract: batch * K = %lld exceeds the 32-bit ciphertext index",
              (long long)batch * K);
    return PNB_ERR_INVALID;
  }
  // a null index makes the gather dense: group g reads ciphertexts g*K .. g*K + K-1
  return lwe_contract_gather_placed(W, bias, delta, M, K, X, nullptr, batch, Y, L, 0, st, ldx,
                                    ldy);
}

}  // namespace pnb
