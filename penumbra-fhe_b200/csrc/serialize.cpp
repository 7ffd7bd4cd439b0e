// serialize.cpp -- byte containers for key sets and LWE ciphertext batches.
//
// The reference generates its keys in-process (runtime/src/keys.rs:47-56) and serialises
// nothing; these containers let a client ship evaluation keys and ciphertexts to a server that
// holds no secrets.  Layout (little-endian, every section 8-byte aligned):
//
//   key set:     "PNBK" u32 version | pnb_params (56 bytes) | u32 flags (bit 0: secret keys
//                present) | u32 reserved | [lwe_sk n][glwe_sk kN] u64 (flags & 1) |
//                bsk u64 [n][(k+1) l][k+1][N] (standard domain) | ksk u64 [kN][ks_level][n+1]
//   ciphertexts: "PNBC" u32 version | u32 count | u32 dim | count x (dim + 1) u64, body last
//
// The arrays are the layouts pnb_keys_export / pnb_keys_import use; the ciphertext rows are
// LWE ciphertexts as the C ABI holds them (mask then body).
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/penumbra_b200.h"

namespace pnb {
void set_error(const char* fmt, ...);  // the library's thread-local last error (capi.cu)
}
using pnb::set_error;

namespace {

constexpr uint32_t KEYS_MAGIC = 0x4b424e50u;  // "PNBK"
constexpr uint32_t CT_MAGIC = 0x43424e50u;    // "PNBC"
constexpr uint32_t VERSION = 1;
constexpr size_t KEYS_HEADER = 8 + sizeof(pnb_params) + 8;
constexpr size_t CT_HEADER = 16;

struct Sizes {
  size_t lwe_sk, glwe_sk, bsk, ksk;
};

Sizes sizes_of(const pnb_params& p) {
  Sizes z;
  z.lwe_sk = (size_t)p.n;
  z.glwe_sk = (size_t)p.k * p.N;
  z.bsk = (size_t)p.n * (p.k + 1) * p.pbs_level * (p.k + 1) * p.N;
  z.ksk = (size_t)p.k * p.N * p.ks_level * (p.n + 1);
  return z;
}

void put32(unsigned char* b, uint32_t v) { memcpy(b, &v, 4); }
uint32_t get32(const unsigned char* b) {
  uint32_t v;
  memcpy(&v, b, 4);
  return v;
}

}  // namespace

extern "C" {

size_t pnb_keys_serialized_bytes(const pnb_keys* keys, int with_secrets) {
  pnb_params p;
  int dev = 0;
  size_t fb = 0, kb = 0;
  if (!keys || pnb_keys_info(keys, &p, &dev, &fb, &kb) != PNB_OK) return 0;
  const Sizes z = sizes_of(p);
  return KEYS_HEADER + 8 * ((with_secrets ? z.lwe_sk + z.glwe_sk : 0) + z.bsk + z.ksk);
}

int pnb_keys_serialize(const pnb_keys* keys, int with_secrets, void* out_host, size_t cap) {
  pnb_params p;
  int dev = 0;
  size_t fb = 0, kb = 0;
  if (!keys || !out_host) {
    set_error("pnb_keys_serialize: NULL argument");
    return PNB_ERR_INVALID;
  }
  int rc = pnb_keys_info(keys, &p, &dev, &fb, &kb);
  if (rc) return rc;
  const size_t need = pnb_keys_serialized_bytes(keys, with_secrets);
  if (cap < need) {
    set_error("pnb_keys_serialize: %zu bytes needed, the buffer holds %zu", need, cap);
    return PNB_ERR_INVALID;
  }
  const Sizes z = sizes_of(p);
  unsigned char* b = static_cast<unsigned char*>(out_host);
  put32(b, KEYS_MAGIC);
  put32(b + 4, VERSION);
  memcpy(b + 8, &p, sizeof p);
  put32(b + 8 + sizeof p, with_secrets ? 1u : 0u);
  put32(b + 12 + sizeof p, 0u);
  uint64_t* w = reinterpret_cast<uint64_t*>(b + KEYS_HEADER);
  uint64_t* lwe = with_secrets ? w : nullptr;
  uint64_t* glwe = with_secrets ? w + z.lwe_sk : nullptr;
  uint64_t* bsk = w + (with_secrets ? z.lwe_sk + z.glwe_sk : 0);
  uint64_t* ksk = bsk + z.bsk;
  return pnb_keys_export(keys, lwe, glwe, bsk, ksk);
}

int pnb_keys_deserialize(int device, const void* in_host, size_t len, pnb_keys** out) {
  if (!in_host || !out || len < KEYS_HEADER) {
    set_error("pnb_keys_deserialize: NULL argument or a buffer shorter than the header");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  const unsigned char* b = static_cast<const unsigned char*>(in_host);
  if (get32(b) != KEYS_MAGIC || get32(b + 4) != VERSION) {
    set_error("pnb_keys_deserialize: not a version-%u key-set container", VERSION);
    return PNB_ERR_INVALID;
  }
  pnb_params p;
  memcpy(&p, b + 8, sizeof p);
  const uint32_t flags = get32(b + 8 + sizeof p);
  if (p.n <= 0 || p.k <= 0 || p.N <= 0 || p.pbs_level <= 0 || p.ks_level <= 0 ||
      p.n > (1 << 16) || p.N > (1 << 16) || p.pbs_level > 64 || p.ks_level > 64) {
    set_error("pnb_keys_deserialize: implausible parameters in the header");
    return PNB_ERR_INVALID;
  }
  const Sizes z = sizes_of(p);
  const bool sec = (flags & 1u) != 0;
  const size_t need = KEYS_HEADER + 8 * ((sec ? z.lwe_sk + z.glwe_sk : 0) + z.bsk + z.ksk);
  if (len < need) {
    set_error("pnb_keys_deserialize: %zu bytes given, the header describes %zu", len, need);
    return PNB_ERR_INVALID;
  }
  // copy to an aligned buffer (the caller's bytes may sit at any address)
  std::vector<uint64_t> w((need - KEYS_HEADER) / 8);
  memcpy(w.data(), b + KEYS_HEADER, need - KEYS_HEADER);
  const uint64_t* lwe = sec ? w.data() : nullptr;
  const uint64_t* glwe = sec ? w.data() + z.lwe_sk : nullptr;
  const uint64_t* bsk = w.data() + (sec ? z.lwe_sk + z.glwe_sk : 0);
  const uint64_t* ksk = bsk + z.bsk;
  return pnb_keys_import(device, &p, lwe, glwe, bsk, ksk, out);
}

size_t pnb_lwe_serialized_bytes(int count, int dim) {
  if (count < 0 || dim < 0) return 0;
  return CT_HEADER + 8 * (size_t)count * ((size_t)dim + 1);
}

int pnb_lwe_serialize(const uint64_t* ct_host, int count, int dim, void* out_host, size_t cap) {
  if ((!ct_host && count > 0) || !out_host || count < 0 || dim < 0) {
    set_error("pnb_lwe_serialize: bad argument");
    return PNB_ERR_INVALID;
  }
  const size_t need = pnb_lwe_serialized_bytes(count, dim);
  if (cap < need) {
    set_error("pnb_lwe_serialize: %zu bytes needed, the buffer holds %zu", need, cap);
    return PNB_ERR_INVALID;
  }
  unsigned char* b = static_cast<unsigned char*>(out_host);
  put32(b, CT_MAGIC);
  put32(b + 4, VERSION);
  put32(b + 8, (uint32_t)count);
  put32(b + 12, (uint32_t)dim);
  if (count > 0) memcpy(b + CT_HEADER, ct_host, need - CT_HEADER);
  return PNB_OK;
}

int pnb_lwe_deserialize(const void* in_host, size_t len, uint64_t* ct_host, size_t cap_words,
                        int* count, int* dim) {
  if (!in_host || !count || !dim || len < CT_HEADER) {
    set_error("pnb_lwe_deserialize: NULL argument or a buffer shorter than the header");
    return PNB_ERR_INVALID;
  }
  const unsigned char* b = static_cast<const unsigned char*>(in_host);
  if (get32(b) != CT_MAGIC || get32(b + 4) != VERSION) {
    set_error("pnb_lwe_deserialize: not a version-%u ciphertext container", VERSION);
    return PNB_ERR_INVALID;
  }
  const uint32_t c = get32(b + 8), d = get32(b + 12);
  if (c > (uint32_t)INT32_MAX || d > (uint32_t)INT32_MAX) {
    set_error("pnb_lwe_deserialize: implausible count or dimension");
    return PNB_ERR_INVALID;
  }
  const size_t words = (size_t)c * ((size_t)d + 1);
  if (len < CT_HEADER + 8 * words) {
    set_error("pnb_lwe_deserialize: %zu bytes given, the header describes %zu", len,
              CT_HEADER + 8 * words);
    return PNB_ERR_INVALID;
  }
  *count = (int)c;
  *dim = (int)d;
  if (!ct_host) return PNB_OK;  // size query
  if (cap_words < words) {
    set_error("pnb_lwe_deserialize: %zu words needed, the buffer holds %zu", words, cap_words);
    return PNB_ERR_INVALID;
  }
  memcpy(ct_host, b + CT_HEADER, 8 * words);
  return PNB_OK;
}

}  // extern "C"
