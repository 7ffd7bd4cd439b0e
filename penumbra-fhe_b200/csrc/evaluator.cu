// evaluator.cu -- batched execution of a compiled graph program on one GPU, and the graph /
// plan / evaluator entry points of the C ABI.
//
// Replaces the reference's per-sample node walk (runtime/src/eval.rs:86-166): the program built
// by plan.cpp runs once per chunk of samples, every instruction over the whole chunk.  Buffers
// are [sample][element][pitch] u64 big-key LWE ciphertexts of kN+1 words, the pitch rounded up to
// an even number of words so that every row starts 16-byte aligned (the contraction then reads
// its operand by TMA tiles or 16-byte copies); the per-element tables (weights, gather indices,
// linear-combination coefficients, test-vector choices) are uploaded once.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "pnb_internal.cuh"
#include "pnb_keys.h"
#include "plan.hpp"

struct pnb_graph {
  pnb::ir::Graph g;
};

struct pnb_plan {
  pnb::plan::Program prog;
  pnb_params params;
};

struct pnb_keyring {
  int device = 0;
  pnb_params params{};
  std::vector<pnb::plan::KeyLevel> levels;  // the planner's key-set menu for params
  std::vector<pnb_keys*> keys;              // one per level: same secret keys and KSK
};

namespace pnb {
namespace {

constexpr int LIN_TERMS = 4;
constexpr int64_t PBS_SLICE = 1 << 16;  // ciphertexts per keyswitch / rotation launch

struct LinArgs {
  uint64_t* dst;
  int64_t E, rows;  // elements per sample, rows = batch * E
  int L, nt;
  int ld;           // row pitch (words) of dst and every source
  const uint64_t* src[LIN_TERMS];
  int64_t srcE[LIN_TERMS];
  const int64_t* coef[LIN_TERMS];
  int64_t coef_u[LIN_TERMS];
  const int32_t* map[LIN_TERMS];
  const uint64_t* cst;
  uint64_t cst_u;
};

// dst[b][e][c] = sum_t coef_t[e] * src_t[b][map_t[e]][c]  (+ cst[e] on the body c = L-1)
__global__ void __launch_bounds__(256) lin_kernel(LinArgs a) {
  const int64_t row = blockIdx.x * 2ll + (threadIdx.x >> 7);
  if (row >= a.rows) return;
  const int64_t b = row / a.E, e = row - b * a.E;
  const uint64_t* s[LIN_TERMS];
  uint64_t k[LIN_TERMS];
#pragma unroll
  for (int t = 0; t < LIN_TERMS; ++t) {
    s[t] = nullptr;
    k[t] = 0;
    if (t < a.nt) {
      const int64_t m = a.map[t] ? a.map[t][e] : e;
      if (m >= 0) {
        s[t] = a.src[t] + ((size_t)b * a.srcE[t] + m) * a.ld;
        k[t] = (uint64_t)(a.coef[t] ? a.coef[t][e] : a.coef_u[t]);
      }
    }
  }
  const uint64_t body = a.cst ? a.cst[e] : a.cst_u;
  uint64_t* d = a.dst + (size_t)row * a.ld;
  for (int c = threadIdx.x & 127; c < a.L; c += 128) {
    uint64_t v = (c == a.L - 1) ? body : 0;
#pragma unroll
    for (int t = 0; t < LIN_TERMS; ++t)
      if (s[t]) v += k[t] * s[t][c];
    d[c] = v;
  }
}

// Copy `rows` rows of L words per sample between row pitches: dst row (b, e) at
// (b * dst_rows + e) * dst_ld, src row at (b * src_rows + src_off + e) * src_ld.
__global__ void repitch_kernel(uint64_t* __restrict__ dst, int64_t dst_rows, int dst_ld,
                               const uint64_t* __restrict__ src, int64_t src_rows,
                               int64_t src_off, int src_ld, int64_t rows, int batch, int L) {
  const int64_t n = (int64_t)batch * rows;
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t b = r / rows, e = r - b * rows;
    const uint64_t* sp = src + ((size_t)b * src_rows + src_off + e) * src_ld;
    uint64_t* dp = dst + ((size_t)b * dst_rows + e) * dst_ld;
    for (int c = threadIdx.x; c < L; c += blockDim.x) dp[c] = sp[c];
  }
}

// idx[b*P + p][k] = b * Ein + table[p][k]  (-1 stays -1)
__global__ void gather_batch_kernel(const int32_t* table, int P, int K, int64_t Ein, int batch,
                                    int32_t* idx) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t n = (int64_t)batch * P * K;
  if (i >= n) return;
  const int64_t b = i / ((int64_t)P * K), r = i - b * P * K;
  const int32_t v = table[r];
  idx[i] = v < 0 ? -1 : (int32_t)(b * Ein + v);
}

template <typename T>
int upload(const std::vector<T>& v, T** out) {
  *out = nullptr;
  if (v.empty()) return PNB_OK;
  PNB_CUDA(cudaMalloc((void**)out, v.size() * sizeof(T)));
  PNB_CUDA(cudaMemcpy(*out, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return PNB_OK;
}

struct DevInstr {
  // Lin
  const int64_t* coef[LIN_TERMS] = {};
  const int32_t* map[LIN_TERMS] = {};
  const uint64_t* cst = nullptr;
  // Pbs
  const int32_t* tv = nullptr;
  // Contract
  const int8_t* W = nullptr;
  const int64_t* bias = nullptr;
  const int32_t* gather = nullptr;  // per-sample table [P][K]
};

}  // namespace
}  // namespace pnb

struct pnb_evaluator {
  int device = 0;
  pnb_params params{};
  pnb::plan::Program prog;
  std::vector<pnb_keys*> keys;  // per program level (null when unused)
  pnb_keys* client = nullptr;   // the key set whose secret keys encrypt and decrypt
  bool borrowed_keys = false;   // the keys belong to a key ring (pnb_evaluator_create_with)
  std::vector<pnb::DevInstr> dev;
  std::vector<void*> allocations;
  uint64_t* tvs = nullptr;  // [T][N]
  // per-chunk resources
  int chunk = 0;
  std::vector<uint64_t*> bufs;
  std::vector<int32_t*> gathers;  // per instruction: batch-expanded gather index
  uint64_t* small = nullptr;
  void* ks_ws = nullptr;
  size_t ks_ws_bytes = 0;
  int64_t max_pbs_rows = 0;
  int chunk_limit = 1;  // samples per chunk allowed by the memory budget
};

namespace pnb {
namespace {

struct Guard {
  int prev = -1;
  int rc = PNB_OK;
  explicit Guard(int dev) {
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) { rc = cuda_status(e, "cudaGetDevice"); return; }
    if (prev != dev && (e = cudaSetDevice(dev)) != cudaSuccess) rc = cuda_status(e, "cudaSetDevice");
  }
  ~Guard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

void free_chunk(pnb_evaluator* ev) {
  for (auto* p : ev->bufs) cudaFree(p);
  for (auto* p : ev->gathers) cudaFree(p);
  ev->bufs.clear();
  ev->gathers.clear();
  cudaFree(ev->small);
  cudaFree(ev->ks_ws);
  ev->small = nullptr;
  ev->ks_ws = nullptr;
  ev->chunk = 0;
}

int64_t row_words(const pnb_params& p) { return (int64_t)p.k * p.N + 1; }
// Internal row pitch: kN+1 rounded up to an even number of words (16-byte aligned rows).
int64_t row_pitch(const pnb_params& p) { return (row_words(p) + 1) & ~(int64_t)1; }

int alloc_chunk(pnb_evaluator* ev, int chunk) {
  free_chunk(ev);
  const int64_t LP = row_pitch(ev->params);
  const auto& P = ev->prog;
  ev->bufs.assign(P.bufs.size(), nullptr);
  for (size_t i = 0; i < P.bufs.size(); ++i)
    PNB_CUDA(cudaMalloc((void**)&ev->bufs[i], (size_t)chunk * P.bufs[i].elems * LP * 8));
  ev->gathers.assign(P.code.size(), nullptr);
  int64_t max_rows = 0;
  for (size_t i = 0; i < P.code.size(); ++i) {
    const auto& I = P.code[i];
    if (I.kind == plan::Kind::Pbs)
      max_rows = std::max<int64_t>(max_rows, (int64_t)chunk * P.bufs[I.dst].elems);
    if (I.kind == plan::Kind::Contract && !I.gather.empty()) {
      const int64_t n = (int64_t)chunk * I.P * I.K;
      PNB_CUDA(cudaMalloc((void**)&ev->gathers[i], n * sizeof(int32_t)));
      gather_batch_kernel<<<(unsigned)((n + 255) / 256), 256>>>(
          ev->dev[i].gather, I.P, I.K, P.bufs[I.src].elems, chunk, ev->gathers[i]);
      PNB_CHECK_LAUNCH("gather_batch_kernel");
    }
  }
  ev->max_pbs_rows = std::min<int64_t>(max_rows, PBS_SLICE);
  if (ev->max_pbs_rows > 0) {
    const pnb_keys* K0 = ev->client;
    PNB_CUDA(cudaMalloc((void**)&ev->small,
                        (size_t)ev->max_pbs_rows * (K0->p.n + 1) * sizeof(uint64_t)));
    ev->ks_ws_bytes = ks_tc_workspace_bytes(K0->p, (int)ev->max_pbs_rows);
    PNB_CUDA(cudaMalloc(&ev->ks_ws, ev->ks_ws_bytes));
  }
  PNB_CUDA(cudaDeviceSynchronize());
  ev->chunk = chunk;
  return PNB_OK;
}

int run_lin(pnb_evaluator* ev, const plan::Instr& I, const DevInstr& D, int batch,
            cudaStream_t st) {
  const auto& P = ev->prog;
  LinArgs a;
  memset(&a, 0, sizeof a);
  a.dst = ev->bufs[I.dst];
  a.E = P.bufs[I.dst].elems;
  a.rows = (int64_t)batch * a.E;
  a.L = (int)row_words(ev->params);
  a.ld = (int)row_pitch(ev->params);
  a.nt = (int)I.terms.size();
  if (a.nt > LIN_TERMS) {
    set_error("internal: linear combination with %d terms", a.nt);
    return PNB_ERR_INVALID;
  }
  for (int t = 0; t < a.nt; ++t) {
    const auto& T = I.terms[t];
    a.src[t] = ev->bufs[T.src];
    a.srcE[t] = P.bufs[T.src].elems;
    a.coef[t] = D.coef[t];
    a.coef_u[t] = T.coef.size() == 1 ? T.coef[0] : 0;
    a.map[t] = D.map[t];
  }
  a.cst = D.cst;
  a.cst_u = I.cst.size() == 1 ? I.cst[0] : 0;
  if (a.rows == 0) return PNB_OK;
  lin_kernel<<<(unsigned)((a.rows + 1) / 2), 256, 0, st>>>(a);
  PNB_CHECK_LAUNCH("lin_kernel");
  return PNB_OK;
}

int run_pbs(pnb_evaluator* ev, const plan::Instr& I, const DevInstr& D, int batch,
            cudaStream_t st) {
  const auto& P = ev->prog;
  const int64_t E = P.bufs[I.dst].elems;
  const int64_t rows = (int64_t)batch * E;
  const int L = (int)row_words(ev->params);
  const int LP = (int)row_pitch(ev->params);
  // stage the bootstrap input 2^shift * src + offset in the destination buffer
  LinArgs a;
  memset(&a, 0, sizeof a);
  a.dst = ev->bufs[I.dst];
  a.E = E;
  a.rows = rows;
  a.L = L;
  a.ld = LP;
  a.nt = 1;
  a.src[0] = ev->bufs[I.src];
  a.srcE[0] = P.bufs[I.src].elems;
  a.coef_u[0] = (int64_t)((uint64_t)1 << I.shift);
  a.cst_u = I.offset;
  if (rows == 0) return PNB_OK;
  lin_kernel<<<(unsigned)((rows + 1) / 2), 256, 0, st>>>(a);
  PNB_CHECK_LAUNCH("lin_kernel(bootstrap input)");
  const pnb_keys* K = ev->keys[I.level];
  for (int64_t r0 = 0; r0 < rows; r0 += ev->max_pbs_rows) {
    const int cnt = (int)std::min<int64_t>(ev->max_pbs_rows, rows - r0);
    uint64_t* x = ev->bufs[I.dst] + (size_t)r0 * LP;
    int rc = keyswitch_launch(ev->client, x, ev->small, cnt, ev->ks_ws, st, LP);
    if (rc) return rc;
    // row r of the slice is element (r0 + r) % E of its sample
    rc = blind_rotate_sel(K, ev->tvs, D.tv, (int)E, (int)(r0 % E), ev->small, x, cnt, st, LP);
    if (rc) return rc;
  }
  return PNB_OK;
}

int run_contract(pnb_evaluator* ev, size_t i, const plan::Instr& I, const DevInstr& D,
                 int batch, cudaStream_t st) {
  const int L = (int)row_words(ev->params);
  const int LP = (int)row_pitch(ev->params);
  if (I.gather.empty())
    return lwe_contract_tc(D.W, D.bias, I.bias_delta, I.M, I.K, ev->bufs[I.src],
                           ev->bufs[I.dst], batch, L, st, LP, LP);
  return lwe_contract_gather_placed(D.W, D.bias, I.bias_delta, I.M, I.K, ev->bufs[I.src],
                                    ev->gathers[i], batch * I.P, ev->bufs[I.dst], L, I.P, st,
                                    LP, LP);
}

}  // namespace
}  // namespace pnb

namespace pnb {
namespace {
int evaluator_finish(pnb_evaluator* ev, const pnb_plan* p, size_t max_bytes);
}  // namespace
}  // namespace pnb

using namespace pnb;

extern "C" {

int pnb_graph_load(const char* json, size_t len, pnb_graph** out) {
  if (!json || !out) {
    set_error("pnb_graph_load: NULL argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  try {
    pnb_graph* g = new pnb_graph;
    try {
      g->g = ir::parse_graph(json, len);
      for (const auto& n : g->g.nodes) ir::validate_op(n.op);
    } catch (...) {
      delete g;
      throw;
    }
    *out = g;
    return PNB_OK;
  } catch (const std::bad_alloc&) {
    set_error("pnb_graph_load: out of host memory");
    return PNB_ERR_OOM;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_graph_free(pnb_graph* g) {
  delete g;
  return PNB_OK;
}

int pnb_graph_info(const pnb_graph* g, int* num_nodes, int* num_blocks, int* input_bits) {
  if (!g) {
    set_error("pnb_graph_info: NULL graph");
    return PNB_ERR_INVALID;
  }
  if (num_nodes) *num_nodes = (int)g->g.nodes.size();
  if (num_blocks) *num_blocks = g->g.num_blocks;
  if (input_bits) *input_bits = g->g.input_bits;
  return PNB_OK;
}

int pnb_graph_check_budget(const pnb_graph* g) {
  if (!g) {
    set_error("pnb_graph_check_budget: NULL graph");
    return PNB_ERR_INVALID;
  }
  try {
    ir::check_graph_bit_width_budget(g->g);
    return PNB_OK;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_op_bits(const char* op_json, size_t len, const int* input_bits, int n_inputs,
                int* output_bits, int* internal_bits) {
  if (!op_json || (!input_bits && n_inputs > 0) || n_inputs < 0 || !output_bits ||
      !internal_bits) {
    set_error("pnb_op_bits: bad argument");
    return PNB_ERR_INVALID;
  }
  try {
    ir::op_bits(op_json, len, std::vector<int>(input_bits, input_bits + n_inputs), output_bits,
                internal_bits);
    return PNB_OK;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_plan_create(const pnb_graph* g, const pnb_params* p, const int64_t* input_lens,
                    int64_t input_lo, int64_t input_hi, double margin_sigmas, pnb_plan** out) {
  if (!g || !p || !out) {
    set_error("pnb_plan_create: NULL argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  try {
    plan::Options o;
    o.input_lo = input_lo;
    o.input_hi = input_hi;
    if (margin_sigmas > 0) o.z = margin_sigmas;
    o.n = p->n;
    o.N = p->N;
    o.log2_ksms = plan::ksms_log2_sigma(p->n, p->N, p->k, p->ks_base_log, p->ks_level, p->lwe_std);
    o.log2_fresh = std::log2(p->glwe_std) + 64;
    o.levels = plan::default_levels(p->n, p->N, p->k, p->glwe_std);
    if (input_lens) o.input_lens.assign(input_lens, input_lens + g->g.inputs.size());
    pnb_plan* pl = new pnb_plan;
    try {
      pl->prog = plan::build(g->g, o);
    } catch (...) {
      delete pl;
      throw;
    }
    pl->params = *p;
    *out = pl;
    return PNB_OK;
  } catch (const std::bad_alloc&) {
    set_error("pnb_plan_create: out of host memory");
    return PNB_ERR_OOM;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_plan_free(pnb_plan* p) {
  delete p;
  return PNB_OK;
}

int pnb_plan_info(const pnb_plan* p, pnb_plan_summary* info) {
  if (!p || !info) {
    set_error("pnb_plan_info: NULL argument");
    return PNB_ERR_INVALID;
  }
  const auto& P = p->prog;
  info->input_elems = P.input_elems;
  info->output_elems = P.output_elems;
  info->num_inputs = (int)P.inputs.size();
  info->num_outputs = (int)P.outputs.size();
  info->pbs_per_sample = P.pbs_per_sample;
  info->cost_per_sample = P.cost_per_sample;
  info->num_instructions = (int)P.code.size();
  return PNB_OK;
}

int pnb_plan_tensor(const pnb_plan* p, int is_output, int idx, int64_t* elems, int* scale_log2,
                    int64_t* lo, int64_t* hi) {
  if (!p) {
    set_error("pnb_plan_tensor: NULL plan");
    return PNB_ERR_INVALID;
  }
  const auto& v = is_output ? p->prog.outputs : p->prog.inputs;
  if (idx < 0 || idx >= (int)v.size()) {
    set_error("pnb_plan_tensor: index %d out of range (%zu tensors)", idx, v.size());
    return PNB_ERR_INVALID;
  }
  if (elems) *elems = v[idx].elems;
  if (scale_log2) *scale_log2 = v[idx].scale;
  if (lo) *lo = v[idx].lo;
  if (hi) *hi = v[idx].hi;
  return PNB_OK;
}

int pnb_plan_key_sets(const pnb_plan* p, int cap, int* base_log, int* level, int64_t* count) {
  if (!p || cap < 0) {
    set_error("pnb_plan_key_sets: bad argument");
    return -1;
  }
  const auto& P = p->prog;
  int n = 0;
  for (size_t l = 0; l < P.pbs_per_level.size(); ++l) {
    if (!P.pbs_per_level[l]) continue;
    if (n < cap) {
      if (base_log) base_log[n] = P.levels[l].base_log;
      if (level) level[n] = P.levels[l].level;
      if (count) count[n] = P.pbs_per_level[l];
    }
    ++n;
  }
  return n;
}

size_t pnb_plan_report(const pnb_plan* p, char* buf, size_t cap) {
  if (!p) return 0;
  const std::string& r = p->prog.report;
  if (buf && cap > 0) {
    const size_t n = std::min(cap - 1, r.size());
    memcpy(buf, r.data(), n);
    buf[n] = 0;
  }
  return r.size() + 1;
}

int pnb_plan_simulate(const pnb_plan* p, const int64_t* inputs, int batch, int64_t* outputs,
                      double* min_margin) {
  if (!p || !inputs || !outputs || batch < 0) {
    set_error("pnb_plan_simulate: bad argument");
    return PNB_ERR_INVALID;
  }
  try {
    plan::simulate(p->prog, inputs, batch, outputs, min_margin);
    return PNB_OK;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_evaluator_free(pnb_evaluator* ev) {
  if (!ev) return PNB_OK;
  Guard g(ev->device);
  free_chunk(ev);
  for (void* a : ev->allocations) cudaFree(a);
  cudaFree(ev->tvs);
  if (!ev->borrowed_keys)
    for (pnb_keys* k : ev->keys)
      if (k) pnb_keys_free(k);
  delete ev;
  return PNB_OK;
}

int pnb_evaluator_create(const pnb_plan* p, int device, uint64_t seed, size_t max_bytes,
                         pnb_evaluator** out) {
  if (!p || !out) {
    set_error("pnb_evaluator_create: NULL argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  Guard guard(device);
  if (guard.rc) return guard.rc;
  pnb_evaluator* ev = new (std::nothrow) pnb_evaluator;
  if (!ev) {
    set_error("pnb_evaluator_create: out of host memory");
    return PNB_ERR_OOM;
  }
  ev->device = device;
  ev->params = p->params;
  ev->prog = p->prog;
  const auto& P = ev->prog;
  int rc = PNB_OK;
  // key sets: one per bootstrap level the program uses (same seed: same secret keys and KSK)
  std::vector<char> used(P.levels.size(), 0);
  for (const auto& I : P.code)
    if (I.kind == plan::Kind::Pbs) used[I.level] = 1;
  ev->keys.assign(P.levels.size(), nullptr);
  for (size_t l = 0; l < P.levels.size() && rc == PNB_OK; ++l) {
    if (!used[l] && !(l == 0 && ev->client == nullptr)) continue;
    pnb_params q = p->params;
    q.pbs_base_log = P.levels[l].base_log;
    q.pbs_level = P.levels[l].level;
    rc = pnb_keygen(device, &q, seed, &ev->keys[l]);
    if (rc == PNB_OK && !ev->client) ev->client = ev->keys[l];
  }
  if (rc == PNB_OK && !ev->client) {
    pnb_params q = p->params;
    rc = pnb_keygen(device, &q, seed, &ev->keys[0]);
    ev->client = ev->keys[0];
  }
  if (rc == PNB_OK) rc = evaluator_finish(ev, p, max_bytes);
  if (rc != PNB_OK) {
    pnb_evaluator_free(ev);
    return rc;
  }
  *out = ev;
  return PNB_OK;
}

int pnb_keyring_create(int device, const pnb_params* params, uint64_t seed, pnb_keyring** out) {
  if (!params || !out) {
    set_error("pnb_keyring_create: NULL argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  pnb_keyring* r = new (std::nothrow) pnb_keyring;
  if (!r) {
    set_error("pnb_keyring_create: out of host memory");
    return PNB_ERR_OOM;
  }
  r->device = device;
  r->params = *params;
  r->levels = plan::default_levels(params->n, params->N, params->k, params->glwe_std);
  r->keys.assign(r->levels.size(), nullptr);
  int rc = PNB_OK;
  for (size_t l = 0; l < r->levels.size() && rc == PNB_OK; ++l) {
    pnb_params q = *params;
    q.pbs_base_log = r->levels[l].base_log;
    q.pbs_level = r->levels[l].level;
    rc = pnb_keygen(device, &q, seed, &r->keys[l]);
  }
  if (rc != PNB_OK) {
    pnb_keyring_free(r);
    return rc;
  }
  *out = r;
  return PNB_OK;
}

int pnb_keyring_free(pnb_keyring* r) {
  if (!r) return PNB_OK;
  for (pnb_keys* k : r->keys)
    if (k) pnb_keys_free(k);
  delete r;
  return PNB_OK;
}

int pnb_keyring_keys(const pnb_keyring* r, int idx, pnb_keys** keys) {
  if (!r || !keys || idx < 0 || idx >= (int)r->keys.size()) {
    set_error("pnb_keyring_keys: bad argument (index %d of %d key sets)", idx,
              r ? (int)r->keys.size() : 0);
    return PNB_ERR_INVALID;
  }
  *keys = r->keys[idx];
  return PNB_OK;
}

int pnb_evaluator_create_with(const pnb_plan* p, const pnb_keyring* ring, size_t max_bytes,
                              pnb_evaluator** out) {
  if (!p || !ring || !out) {
    set_error("pnb_evaluator_create_with: NULL argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  const pnb_params& a = p->params;
  const pnb_params& b = ring->params;
  if (a.n != b.n || a.k != b.k || a.N != b.N || a.ks_base_log != b.ks_base_log ||
      a.ks_level != b.ks_level || a.lwe_std != b.lwe_std || a.glwe_std != b.glwe_std) {
    set_error("pnb_evaluator_create_with: the plan was compiled for another parameter set than "
              "the key ring's");
    return PNB_ERR_INVALID;
  }
  const auto& P = p->prog;
  if (P.levels.size() != ring->levels.size()) {
    set_error("pnb_evaluator_create_with: the plan's key-set menu differs from the key ring's");
    return PNB_ERR_INVALID;
  }
  for (size_t l = 0; l < P.levels.size(); ++l)
    if (P.levels[l].base_log != ring->levels[l].base_log ||
        P.levels[l].level != ring->levels[l].level) {
      set_error("pnb_evaluator_create_with: the plan's key-set menu differs from the key ring's");
      return PNB_ERR_INVALID;
    }
  Guard guard(ring->device);
  if (guard.rc) return guard.rc;
  pnb_evaluator* ev = new (std::nothrow) pnb_evaluator;
  if (!ev) {
    set_error("pnb_evaluator_create_with: out of host memory");
    return PNB_ERR_OOM;
  }
  ev->device = ring->device;
  ev->params = p->params;
  ev->prog = p->prog;
  ev->keys = ring->keys;
  ev->borrowed_keys = true;
  ev->client = ring->keys[0];
  int rc = evaluator_finish(ev, p, max_bytes);
  if (rc != PNB_OK) {
    pnb_evaluator_free(ev);
    return rc;
  }
  *out = ev;
  return PNB_OK;
}

}  // extern "C"

namespace pnb {
namespace {

// Test vectors, per-instruction tables and the chunk limit of an evaluator whose key sets are
// in place.
int evaluator_finish(pnb_evaluator* ev, const pnb_plan* p, size_t max_bytes) {
  const auto& P = ev->prog;
  int rc = PNB_OK;
  // test vectors
  const int N = p->params.N;
  if (rc == PNB_OK && !P.tvs.empty()) {
    std::vector<uint64_t> t;
    for (const auto& s : P.tvs) {
      std::vector<uint64_t> m = plan::materialize_tv(s, N);
      t.insert(t.end(), m.begin(), m.end());
    }
    rc = upload(t, &ev->tvs);
  }
  // per-instruction tables
  ev->dev.assign(P.code.size(), DevInstr{});
  auto keep = [&](void* a) {
    if (a) ev->allocations.push_back(a);
  };
  for (size_t i = 0; i < P.code.size() && rc == PNB_OK; ++i) {
    const auto& I = P.code[i];
    DevInstr& D = ev->dev[i];
    if (I.kind == plan::Kind::Lin) {
      for (size_t t = 0; t < I.terms.size() && rc == PNB_OK; ++t) {
        int64_t* c = nullptr;
        int32_t* m = nullptr;
        if (I.terms[t].coef.size() > 1) rc = upload(I.terms[t].coef, &c);
        if (rc == PNB_OK) rc = upload(I.terms[t].map, &m);
        keep(c);
        keep(m);
        D.coef[t] = c;
        D.map[t] = m;
      }
      uint64_t* c = nullptr;
      if (rc == PNB_OK && I.cst.size() > 1) rc = upload(I.cst, &c);
      keep(c);
      D.cst = c;
    } else if (I.kind == plan::Kind::Pbs) {
      int32_t* t = nullptr;
      std::vector<int32_t> idx = I.tv;
      if (idx.size() == 1) idx.assign((size_t)P.bufs[I.dst].elems, I.tv[0]);
      rc = upload(idx, &t);
      keep(t);
      D.tv = t;
    } else {
      int8_t* w = nullptr;
      int64_t* b = nullptr;
      int32_t* gt = nullptr;
      rc = upload(I.W, &w);
      if (rc == PNB_OK) rc = upload(I.bias, &b);
      if (rc == PNB_OK) rc = upload(I.gather, &gt);
      keep(w);
      keep(b);
      keep(gt);
      D.W = w;
      D.bias = b;
      D.gather = gt;
    }
  }
  if (rc == PNB_OK) {
    // chunk size: as many samples as fit the memory budget
    int64_t per_sample = 0;
    for (const auto& b : P.bufs) per_sample += b.elems * row_pitch(p->params) * 8;
    size_t budget = max_bytes;
    if (budget == 0) {
      size_t fr = 0, tot = 0;
      cudaMemGetInfo(&fr, &tot);
      budget = fr / 2;
    }
    // the per-chunk buffers are allocated by the first evaluate (sized by its batch)
    ev->chunk_limit = (int)std::max<int64_t>(
        1, std::min<int64_t>(1 << 20, (int64_t)budget / std::max<int64_t>(per_sample, 1)));
  }
  return rc;
}

}  // namespace
}  // namespace pnb

extern "C" {

int pnb_evaluator_keys(const pnb_evaluator* ev, pnb_keys** keys) {
  if (!ev || !keys) {
    set_error("pnb_evaluator_keys: NULL argument");
    return PNB_ERR_INVALID;
  }
  *keys = ev->client;
  return PNB_OK;
}

int pnb_evaluator_reserve(pnb_evaluator* ev, int batch) {
  if (!ev || batch < 0) {
    set_error("pnb_evaluator_reserve: bad argument");
    return PNB_ERR_INVALID;
  }
  Guard guard(ev->device);
  if (guard.rc) return guard.rc;
  const int want = std::min(batch, ev->chunk_limit);
  return ev->chunk < want ? alloc_chunk(ev, want) : PNB_OK;
}

int pnb_evaluate(pnb_evaluator* ev, const uint64_t* in_dev, int batch, uint64_t* out_dev,
                 void* stream) {
  if (!ev || batch < 0 || (batch > 0 && (!in_dev || !out_dev))) {
    set_error("pnb_evaluate: bad argument");
    return PNB_ERR_INVALID;
  }
  if (batch == 0) return PNB_OK;
  Guard guard(ev->device);
  if (guard.rc) return guard.rc;
  cudaStream_t st = (cudaStream_t)stream;
  const auto& P = ev->prog;
  const int64_t L = row_words(ev->params);
  int rc = PNB_OK;
  const int want = std::min(batch, ev->chunk_limit);
  if (ev->chunk < want) rc = alloc_chunk(ev, want);
  if (rc) return rc;
  const int chunk = ev->chunk;
  for (int b0 = 0; b0 < batch && rc == PNB_OK; b0 += chunk) {
    const int nb = std::min(chunk, batch - b0);
    const int LP = (int)row_pitch(ev->params);
    auto grid_of = [](int64_t rows) { return (unsigned)std::min<int64_t>(rows, 148 * 32); };
    int64_t off = 0;
    for (const auto& io : P.inputs) {
      repitch_kernel<<<grid_of((int64_t)nb * io.elems), 256, 0, st>>>(
          ev->bufs[io.buf], io.elems, LP, in_dev + (size_t)b0 * P.input_elems * L,
          P.input_elems, off, (int)L, io.elems, nb, (int)L);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_status(e, "pnb_evaluate: input copy");
      off += io.elems;
    }
    for (size_t i = 0; i < P.code.size() && rc == PNB_OK; ++i) {
      const auto& I = P.code[i];
      switch (I.kind) {
        case plan::Kind::Lin: rc = run_lin(ev, I, ev->dev[i], nb, st); break;
        case plan::Kind::Pbs: rc = run_pbs(ev, I, ev->dev[i], nb, st); break;
        case plan::Kind::Contract: rc = run_contract(ev, i, I, ev->dev[i], nb, st); break;
      }
    }
    off = 0;
    for (const auto& io : P.outputs) {
      if (rc) break;
      // output tensor io is columns [off, off + elems) of each sample's output rows
      repitch_kernel<<<grid_of((int64_t)nb * io.elems), 256, 0, st>>>(
          out_dev + ((size_t)b0 * P.output_elems + off) * L, P.output_elems, (int)L,
          ev->bufs[io.buf], io.elems, 0, LP, io.elems, nb, (int)L);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_status(e, "pnb_evaluate: output copy");
      off += io.elems;
    }
  }
  return rc;
}


// ---- one op at a time ------------------------------------------------------------------------

int pnb_op_plan_create(const char* op_json, size_t len, const pnb_params* p,
                       const pnb_tensor_desc* in, int n_inputs, int out_scale_log2,
                       double out_log2_sigma, double margin_sigmas, pnb_plan** out) {
  if (!op_json || !p || !in || n_inputs < 1 || n_inputs > 2 || !out || out_scale_log2 < 0 ||
      out_scale_log2 > 62 || out_log2_sigma < 0) {
    set_error("pnb_op_plan_create: bad argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  try {
    // a one-node graph over inputs x0 (x1) -> y; the op payload is validated by the IR reader
    std::string doc = "{\"schema_version\":\"";
    doc += ir::SCHEMA_VERSION;
    doc += "\",\"num_blocks\":31,\"input_bits\":1,\"inputs\":[\"x0\"";
    if (n_inputs == 2) doc += ",\"x1\"";
    doc += "],\"outputs\":[\"y\"],\"nodes\":[{\"name\":\"op\",\"inputs\":[\"x0\"";
    if (n_inputs == 2) doc += ",\"x1\"";
    doc += "],\"outputs\":[\"y\"],\"op\":";
    doc.append(op_json, len);
    doc += "}]}";
    ir::Graph g = ir::parse_graph(doc.data(), doc.size());
    for (const auto& n : g.nodes) ir::validate_op(n.op);
    plan::Options o;
    o.input_lo = in[0].lo;
    o.input_hi = in[0].hi;
    if (margin_sigmas > 0) o.z = margin_sigmas;
    o.n = p->n;
    o.N = p->N;
    o.log2_ksms = plan::ksms_log2_sigma(p->n, p->N, p->k, p->ks_base_log, p->ks_level, p->lwe_std);
    o.log2_fresh = std::log2(p->glwe_std) + 64;
    o.levels = plan::default_levels(p->n, p->N, p->k, p->glwe_std);
    o.check_budget = false;
    o.output_scale = out_scale_log2;
    o.output_log2_sigma = out_log2_sigma;
    for (int i = 0; i < n_inputs; ++i) {
      if (in[i].elems <= 0) {
        set_error("pnb_op_plan_create: input %d has %lld elements", i, (long long)in[i].elems);
        return PNB_ERR_INVALID;
      }
      o.input_lens.push_back(in[i].elems);
      plan::InputSpec sp;
      sp.scale = in[i].scale_log2;
      sp.log2_sigma = in[i].log2_sigma;
      sp.ranged = true;
      sp.lo = in[i].lo;
      sp.hi = in[i].hi;
      o.input_specs.push_back(sp);
    }
    pnb_plan* pl = new pnb_plan;
    try {
      pl->prog = plan::build(g, o);
    } catch (...) {
      delete pl;
      throw;
    }
    pl->params = *p;
    *out = pl;
    return PNB_OK;
  } catch (const std::bad_alloc&) {
    set_error("pnb_op_plan_create: out of host memory");
    return PNB_ERR_OOM;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_radix_plan_create(const pnb_params* p, int num_blocks, int is_signed, int to_blocks,
                          int block_max, const pnb_tensor_desc* wide, double margin_sigmas,
                          pnb_plan** out) {
  if (!p || !wide || !out || num_blocks < 1 || wide->elems < 1) {
    set_error("pnb_radix_plan_create: bad argument");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  try {
    plan::Options o;
    if (margin_sigmas > 0) o.z = margin_sigmas;
    o.n = p->n;
    o.N = p->N;
    o.log2_ksms = plan::ksms_log2_sigma(p->n, p->N, p->k, p->ks_base_log, p->ks_level, p->lwe_std);
    o.log2_fresh = std::log2(p->glwe_std) + 64;
    o.levels = plan::default_levels(p->n, p->N, p->k, p->glwe_std);
    plan::RadixSpec r;
    r.to_blocks = to_blocks != 0;
    r.is_signed = is_signed != 0;
    r.num_blocks = num_blocks;
    r.msg_bits = p->msg_bits;
    r.carry_bits = p->carry_bits;
    r.block_max = block_max;
    r.elems = wide->elems;
    r.wide.scale = wide->scale_log2;
    r.wide.log2_sigma = wide->log2_sigma;
    r.wide.ranged = true;
    r.wide.lo = wide->lo;
    r.wide.hi = wide->hi;
    pnb_plan* pl = new pnb_plan;
    try {
      pl->prog = plan::build_radix(r, o);
    } catch (...) {
      delete pl;
      throw;
    }
    pl->params = *p;
    *out = pl;
    return PNB_OK;
  } catch (const std::bad_alloc&) {
    set_error("pnb_radix_plan_create: out of host memory");
    return PNB_ERR_OOM;
  } catch (const std::exception& e) {
    set_error("%s", e.what());
    return PNB_ERR_INVALID;
  }
}

int pnb_plan_tensor_desc(const pnb_plan* p, int is_output, int idx, pnb_tensor_desc* d) {
  if (!p || !d) {
    set_error("pnb_plan_tensor_desc: NULL argument");
    return PNB_ERR_INVALID;
  }
  const auto& v = is_output ? p->prog.outputs : p->prog.inputs;
  if (idx < 0 || idx >= (int)v.size()) {
    set_error("pnb_plan_tensor_desc: index %d out of range (%zu tensors)", idx, v.size());
    return PNB_ERR_INVALID;
  }
  memset(d, 0, sizeof *d);
  d->elems = v[idx].elems;
  d->lo = v[idx].lo;
  d->hi = v[idx].hi;
  d->scale_log2 = v[idx].scale;
  d->log2_sigma = v[idx].log2_sigma;
  return PNB_OK;
}

}  // extern "C"

namespace pnb {
namespace {

// Compile one op over `in`, bind it to the ring and run it on `batch` samples, packing several
// inputs into the evaluator's [sample][input elements] layout.  Blocking.
int run_one_op(const pnb_keyring* ring, const std::string& op_json, const pnb_tensor_desc* in,
               const uint64_t* const* in_dev, int n_in, int batch, int out_scale,
               double out_sigma, uint64_t* out_dev, pnb_tensor_desc* out_desc, cudaStream_t st,
               const char* who) {
  if (!ring || !in || !in_dev || !out_dev || batch < 0) {
    set_error("%s: bad argument", who);
    return PNB_ERR_INVALID;
  }
  for (int i = 0; i < n_in; ++i)
    if (!in_dev[i] && batch > 0) {
      set_error("%s: NULL input", who);
      return PNB_ERR_INVALID;
    }
  pnb_plan* pl = nullptr;
  int rc = pnb_op_plan_create(op_json.data(), op_json.size(), &ring->params, in, n_in,
                              out_scale, out_sigma, 0, &pl);
  if (rc) return rc;
  if (out_desc) rc = pnb_plan_tensor_desc(pl, 1, 0, out_desc);
  pnb_evaluator* ev = nullptr;
  if (rc == PNB_OK) rc = pnb_evaluator_create_with(pl, ring, 0, &ev);
  if (rc == PNB_OK && batch > 0) {
    Guard guard(ring->device);
    rc = guard.rc;
    const int64_t L = row_words(ring->params);
    const uint64_t* src = in_dev[0];
    uint64_t* packed = nullptr;
    if (rc == PNB_OK && n_in > 1) {
      // [batch][e0 + e1][L] from the separate input tensors
      int64_t tot = 0;
      for (int i = 0; i < n_in; ++i) tot += in[i].elems;
      cudaError_t e = cudaMallocAsync((void**)&packed, (size_t)batch * tot * L * 8, st);
      if (e != cudaSuccess) rc = cuda_status(e, "cudaMallocAsync(op inputs)");
      int64_t off = 0;
      for (int i = 0; i < n_in && rc == PNB_OK; ++i) {
        e = cudaMemcpy2DAsync(packed + off * L, (size_t)tot * L * 8, in_dev[i],
                              (size_t)in[i].elems * L * 8, (size_t)in[i].elems * L * 8, batch,
                              cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) rc = cuda_status(e, "cudaMemcpy2DAsync(op inputs)");
        off += in[i].elems;
      }
      src = packed;
    }
    if (rc == PNB_OK) rc = pnb_evaluate(ev, src, batch, out_dev, st);
    if (packed) cudaFreeAsync(packed, st);
    if (rc == PNB_OK) {
      cudaError_t e = cudaStreamSynchronize(st);
      if (e != cudaSuccess) rc = cuda_status(e, who);
    }
  }
  pnb_evaluator_free(ev);
  pnb_plan_free(pl);
  return rc;
}

std::string u64_list(const uint64_t* v, int n) {
  std::string s = "[";
  for (int i = 0; i < n; ++i) s += (i ? "," : "") + std::to_string(v[i]);
  return s + "]";
}

}  // namespace
}  // namespace pnb

extern "C" {

int pnb_requant_batch(const pnb_keyring* ring, const pnb_requant_spec* spec,
                      const pnb_tensor_desc* in, const uint64_t* in_dev, int batch,
                      int out_scale_log2, double out_log2_sigma, uint64_t* out_dev,
                      pnb_tensor_desc* out_desc, void* stream) {
  if (!spec || !spec->mult || !spec->round_bias || !spec->shift || spec->channels < 1 ||
      spec->out_bits < 1 || spec->out_bits > 16) {
    set_error("pnb_requant_batch: bad requant spec");
    return PNB_ERR_INVALID;
  }
  const int lut_n = 1 << spec->out_bits;
  std::vector<uint64_t> lut((size_t)lut_n);
  for (int i = 0; i < lut_n; ++i) lut[i] = spec->clamp_lut ? spec->clamp_lut[i] : (uint64_t)i;
  std::string j = "{\"op_type\":\"Requant\",\"out_bits\":" + std::to_string(spec->out_bits) +
                  ",\"clamp_lut\":" + u64_list(lut.data(), lut_n);
  const int C = spec->channels;
  if (C == 1) {
    j += ",\"shift\":" + std::to_string(spec->shift[0]) + ",\"mult\":" +
         std::to_string(spec->mult[0]) + ",\"round_bias\":" + std::to_string(spec->round_bias[0]);
  } else {
    std::vector<uint64_t> sh(spec->shift, spec->shift + C);
    j += ",\"shift\":" + std::to_string(spec->shift[0]) + ",\"mults\":" +
         u64_list(spec->mult, C) + ",\"round_biases\":" + u64_list(spec->round_bias, C) +
         ",\"shifts\":" + u64_list(sh.data(), C) + ",\"channel_size\":" +
         std::to_string(spec->channel_size);
  }
  j += "}";
  const uint64_t* ins[1] = {in_dev};
  return run_one_op(ring, j, in, ins, 1, batch, out_scale_log2, out_log2_sigma, out_dev,
                    out_desc, (cudaStream_t)stream, "pnb_requant_batch");
}

int pnb_argmax_batch(const pnb_keyring* ring, int64_t threshold, const pnb_tensor_desc* in,
                     const uint64_t* in_dev, int batch, int out_scale_log2,
                     double out_log2_sigma, uint64_t* out_dev, pnb_tensor_desc* out_desc,
                     void* stream) {
  const std::string j = "{\"op_type\":\"Argmax\",\"threshold\":" + std::to_string(threshold) + "}";
  const uint64_t* ins[1] = {in_dev};
  return run_one_op(ring, j, in, ins, 1, batch, out_scale_log2, out_log2_sigma, out_dev,
                    out_desc, (cudaStream_t)stream, "pnb_argmax_batch");
}

int pnb_add_batch(const pnb_keyring* ring, const pnb_tensor_desc* a, const uint64_t* a_dev,
                  const pnb_tensor_desc* b, const uint64_t* b_dev, int batch, int out_scale_log2,
                  double out_log2_sigma, uint64_t* out_dev, pnb_tensor_desc* out_desc,
                  void* stream) {
  if (!a || !b) {
    set_error("pnb_add_batch: NULL descriptor");
    return PNB_ERR_INVALID;
  }
  const pnb_tensor_desc d[2] = {*a, *b};
  const uint64_t* ins[2] = {a_dev, b_dev};
  return run_one_op(ring, "{\"op_type\":\"Add\"}", d, ins, 2, batch, out_scale_log2,
                    out_log2_sigma, out_dev, out_desc, (cudaStream_t)stream, "pnb_add_batch");
}

}  // extern "C"
