// radix.cu -- merge of radix-block ciphertexts into one wide LWE ciphertext per integer.
//
// The reference carries every value as a signed radix integer: `num_blocks` shortint blocks,
// block i holding digit i (msg_bits bits, plus carry room) of the two's-complement value
// (`encrypt::encrypt` -> `RadixClientKey::encrypt_signed`, runtime/src/encrypt.rs:20-22;
// decrypted by `decrypt_signed`, runtime/src/encrypt.rs:43-45).  The kernels here hold one
// integer as one wide LWE ciphertext instead.  A merge re-encodes each block by a lookup
// bootstrap whose table is the block's weighted digit, d -> d * 2^(msg_bits * i) * delta_out
// (the most significant block of a signed integer: its digit read as two's complement), and
// sums the bootstrapped blocks.  The scaling happens inside the bootstrap, so every term
// carries fresh bootstrap noise; scaling the input blocks directly would multiply their noise
// by the block weight.
#include <algorithm>
#include <climits>

#include "pnb_internal.cuh"
#include "pnb_keys.h"

namespace pnb {

static size_t radix_align256(size_t b) { return (b + 255) & ~(size_t)255; }

// out[c][j] = sum over blocks i of parts[c][i][j] (mod 2^64); one thread per output word, so
// neighbouring threads read neighbouring words of each block.
__global__ void radix_sum_kernel(const uint64_t* __restrict__ parts, int nb, int L,
                                 size_t words, uint64_t* __restrict__ out) {
  for (size_t x = (size_t)blockIdx.x * blockDim.x + threadIdx.x; x < words;
       x += (size_t)gridDim.x * blockDim.x) {
    const size_t c = x / (size_t)L, j = x % (size_t)L;
    const uint64_t* p = parts + c * (size_t)nb * L + j;
    uint64_t s = 0;
    for (int i = 0; i < nb; ++i) s += p[(size_t)i * L];
    out[x] = s;
  }
}

__global__ void radix_iota_kernel(int32_t* idx, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) idx[i] = i;
}

// Lookup tables of every block, passed by value so that building the test vectors needs no
// host-to-device copy (a copy from pageable host memory would synchronise the stream).
constexpr int RADIX_LUT_WORDS = 1024;
struct RadixLuts {
  uint64_t v[RADIX_LUT_WORDS];  // [block][lut_len]
};

// Test vector of block blockIdx.y: box m of width N / lut_len holds lut[m] * delta_out, rotated
// by half a box, negated past the half torus (the encoding pnb_test_vector builds).
__global__ void radix_tv_kernel(const RadixLuts luts, int lut_len, uint64_t delta_out, int N,
                                uint64_t* __restrict__ tvs) {
  const int i = blockIdx.y;
  const uint64_t* lut = luts.v + i * lut_len;
  const int box = N / lut_len, half = box / 2;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < N; j += gridDim.x * blockDim.x) {
    const int m = (j + half) / box;
    tvs[(size_t)i * N + j] =
        (m < lut_len) ? lut[m] * delta_out : (uint64_t)0 - lut[m - lut_len] * delta_out;
  }
}

// Lookup table of block `i` of `nb`: entry d (digit plus carries) -> its weighted value.
// Unsigned integers and the lower blocks of signed ones keep their carries (d * 2^(mb i)).
// The top block of a signed integer reads its digit as two's complement and drops the carries
// above it, which lie beyond the integer's width.  The merged value then equals
// decrypt_signed's (the blocks' sum reduced to the integer's width and sign-extended) whenever
// the lower blocks' weighted sum stays below the top block's weight -- always for carry-free
// lower blocks, which is how encrypt_signed and every carry-propagating radix op leave them.
void radix_merge_lut(int msg_bits, int carry_bits, int nb, int i, bool is_signed,
                     uint64_t* lut) {
  const int len = 1 << (msg_bits + carry_bits);
  const int64_t mod = (int64_t)1 << msg_bits;
  const uint64_t weight = (uint64_t)1 << (msg_bits * i);
  for (int d = 0; d < len; ++d) {
    if (is_signed && i == nb - 1) {
      const int64_t dm = d % mod;
      const int64_t sd = dm >= mod / 2 ? dm - mod : dm;
      lut[d] = (uint64_t)sd * weight;
    } else {
      lut[d] = (uint64_t)d * weight;
    }
  }
}

int radix_merge(const pnb_keys* K, const uint64_t* blocks, int nb, int count, bool is_signed,
                uint64_t delta_out, uint64_t* out, cudaStream_t st) {
  const int mb = K->p.msg_bits, cb = K->p.carry_bits;
  if (nb < 1 || (long long)nb * mb > 63) {
    set_error("radix_merge: %d blocks of %d message bits exceed a 63-bit integer", nb, mb);
    return PNB_ERR_INVALID;
  }
  if ((long long)count * nb > INT_MAX) {
    set_error("radix_merge: %d integers x %d blocks exceed one launch", count, nb);
    return PNB_ERR_INVALID;
  }
  const int lut_len = 1 << (mb + cb);
  if ((long long)nb * lut_len > RADIX_LUT_WORDS || lut_len > K->p.N) {
    set_error("radix_merge: %d blocks of %d-entry tables exceed the %d table words a call takes",
              nb, lut_len, RADIX_LUT_WORDS);
    return PNB_ERR_INVALID;
  }
  if (count == 0) return PNB_OK;
  const int N = K->p.N, L = K->p.k * N + 1, total = count * nb;
  const size_t tv_b = radix_align256((size_t)nb * N * sizeof(uint64_t));
  const size_t idx_b = radix_align256((size_t)nb * sizeof(int32_t));
  const size_t small_b = radix_align256((size_t)total * (K->p.n + 1) * sizeof(uint64_t));
  const size_t parts_b = radix_align256((size_t)total * L * sizeof(uint64_t));
  const size_t ks_b = ks_tc_workspace_bytes(K->p, total);
  unsigned char* w = nullptr;
  PNB_CUDA(cudaMallocAsync((void**)&w, tv_b + idx_b + small_b + parts_b + ks_b, st));
  uint64_t* tvs = reinterpret_cast<uint64_t*>(w);
  int32_t* idx = reinterpret_cast<int32_t*>(w + tv_b);
  uint64_t* small = reinterpret_cast<uint64_t*>(w + tv_b + idx_b);
  uint64_t* parts = reinterpret_cast<uint64_t*>(w + tv_b + idx_b + small_b);
  void* digits = w + tv_b + idx_b + small_b + parts_b;

  int rc = PNB_OK;
  {
    RadixLuts luts{};
    for (int i = 0; i < nb; ++i)
      radix_merge_lut(mb, cb, nb, i, is_signed, luts.v + (size_t)i * lut_len);
    radix_tv_kernel<<<dim3((N + 255) / 256, nb), 256, 0, st>>>(luts, lut_len, delta_out, N, tvs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_status(e, "radix_tv_kernel");
  }
  if (rc == PNB_OK) {
    radix_iota_kernel<<<1, 64, 0, st>>>(idx, nb);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_status(e, "radix_iota_kernel");
  }
  // block c of the flattened [count][nb] batch is block (c % nb) of its integer
  if (rc == PNB_OK) rc = keyswitch_launch(K, blocks, small, total, digits, st);
  if (rc == PNB_OK) rc = blind_rotate_sel(K, tvs, idx, nb, 0, small, parts, total, st);
  if (rc == PNB_OK) {
    const size_t words = (size_t)count * L;
    const unsigned grid = (unsigned)std::min<size_t>((words + 255) / 256, 148 * 16);
    radix_sum_kernel<<<grid, 256, 0, st>>>(parts, nb, L, words, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_status(e, "radix_sum_kernel");
  }
  cudaError_t e = cudaFreeAsync(w, st);
  if (rc == PNB_OK && e != cudaSuccess) rc = cuda_status(e, "cudaFreeAsync(radix merge)");
  return rc;
}

}  // namespace pnb
