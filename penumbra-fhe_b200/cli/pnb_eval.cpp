// pnb_eval -- evaluate a model.fhe graph under encryption on one GPU, through the C ABI only.
//
//   pnb_eval MODEL INPUTS [--device D] [--seed S] [--simulate] [--report]
//
// MODEL is the IR graph (a model.fhe document, or any JSON document holding it under "graph");
// INPUTS is a JSON document with "inputs": one integer array per sample (the graph inputs'
// elements concatenated in graph order).  The graph is parsed and budget-checked with the
// reference's rules (runtime/src/ir.rs:169-452, runtime/src/eval.rs:237-276), compiled, its key
// sets generated on the GPU, the inputs encrypted, the whole batch evaluated (the batched form of
// runtime/src/eval.rs:86-166) and the outputs decrypted.  Prints {"outputs": [[...], ...]}.
// --simulate runs the compiled program on noise-free phases on the host instead (no GPU).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/penumbra_b200.h"
#include "../csrc/json.hpp"

namespace {

[[noreturn]] void die(const std::string& m) {
  fprintf(stderr, "pnb_eval: %s\n", m.c_str());
  exit(1);
}

void check(int rc, const char* what) {
  if (rc != PNB_OK) die(std::string(what) + ": " + pnb_last_error());
}

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) die(std::string(what) + ": " + cudaGetErrorString(e));
}

std::string slurp(const char* path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) die(std::string("cannot read ") + path);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

}  // namespace

int main(int argc, char** argv) {
  const char* model = nullptr;
  const char* inputs = nullptr;
  int device = 0;
  unsigned long long seed = 1;
  bool simulate = false, report = false;
  for (int i = 1; i < argc; ++i) {
    if (!strcmp(argv[i], "--device") && i + 1 < argc) device = atoi(argv[++i]);
    else if (!strcmp(argv[i], "--seed") && i + 1 < argc) seed = strtoull(argv[++i], nullptr, 10);
    else if (!strcmp(argv[i], "--simulate")) simulate = true;
    else if (!strcmp(argv[i], "--report")) report = true;
    else if (!model) model = argv[i];
    else if (!inputs) inputs = argv[i];
    else die(std::string("unexpected argument ") + argv[i]);
  }
  if (!model || !inputs) die("usage: pnb_eval MODEL INPUTS [--device D] [--seed S] [--simulate]");

  const std::string gtext = slurp(model);
  pnb_graph* graph = nullptr;
  check(pnb_graph_load(gtext.data(), gtext.size(), &graph), "graph");
  check(pnb_graph_check_budget(graph), "bit-width budget");
  int nodes = 0, blocks = 0, input_bits = 0;
  check(pnb_graph_info(graph, &nodes, &blocks, &input_bits), "graph info");

  const std::string itext = slurp(inputs);
  pnb::json::Value idoc;
  try {
    idoc = pnb::json::parse(itext.data(), itext.size());
  } catch (const std::exception& e) {
    die(std::string("inputs: ") + e.what());
  }
  const pnb::json::Value* arr = idoc.get("inputs");
  if (!arr || arr->kind != pnb::json::Value::Array) die("inputs: no \"inputs\" array");
  const int batch = (int)arr->arr.size();

  pnb_params params;
  check(pnb_params_default(&params), "params");
  pnb_plan* plan = nullptr;
  check(pnb_plan_create(graph, &params, nullptr, 0, (1ll << input_bits) - 1, 0.0, &plan), "plan");
  pnb_plan_summary info;
  check(pnb_plan_info(plan, &info), "plan info");
  if (report) {
    std::vector<char> buf(pnb_plan_report(plan, nullptr, 0));
    pnb_plan_report(plan, buf.data(), buf.size());
    fprintf(stderr, "%s", buf.data());
  }

  std::vector<int64_t> x((size_t)batch * info.input_elems);
  for (int b = 0; b < batch; ++b) {
    const auto& row = arr->arr[b].arr;
    if ((int64_t)row.size() != info.input_elems)
      die("inputs: sample " + std::to_string(b) + " has " + std::to_string(row.size()) +
          " values, the graph takes " + std::to_string(info.input_elems));
    for (int64_t e = 0; e < info.input_elems; ++e) {
      const int64_t v = row[e].i;
      if (v < 0 || v > (1ll << input_bits) - 1)
        die("inputs: value " + std::to_string(v) + " outside the declared " +
            std::to_string(input_bits) + "-bit input range");
      x[(size_t)b * info.input_elems + e] = v;
    }
  }
  std::vector<int64_t> y((size_t)batch * info.output_elems);

  if (simulate) {
    check(pnb_plan_simulate(plan, x.data(), batch, y.data(), nullptr), "simulate");
  } else {
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    pnb_evaluator* ev = nullptr;
    check(pnb_evaluator_create(plan, device, seed, 0, &ev), "evaluator");
    pnb_keys* keys = nullptr;
    check(pnb_evaluator_keys(ev, &keys), "keys");
    const int64_t L = (int64_t)params.k * params.N + 1;
    uint64_t *d_in = nullptr, *d_out = nullptr, *d_tmp = nullptr, *d_ph = nullptr;
    int64_t* d_msg = nullptr;
    check_cuda(cudaMalloc(&d_in, (size_t)batch * info.input_elems * L * 8), "cudaMalloc");
    check_cuda(cudaMalloc(&d_out, (size_t)batch * info.output_elems * L * 8), "cudaMalloc");
    check_cuda(cudaMalloc(&d_msg, (size_t)batch * info.input_elems * 8), "cudaMalloc");
    check_cuda(cudaMalloc(&d_tmp, (size_t)batch * info.input_elems * L * 8), "cudaMalloc");
    check_cuda(cudaMalloc(&d_ph, (size_t)batch * info.output_elems * 8), "cudaMalloc");
    // encrypt each input tensor at its scale, then interleave into [sample][element] order
    int64_t off = 0;
    for (int t = 0; t < info.num_inputs; ++t) {
      int64_t elems = 0;
      int scale = 0;
      check(pnb_plan_tensor(plan, 0, t, &elems, &scale, nullptr, nullptr), "input tensor");
      std::vector<int64_t> m((size_t)batch * elems);
      for (int b = 0; b < batch; ++b)
        for (int64_t e = 0; e < elems; ++e)
          m[(size_t)b * elems + e] = x[(size_t)b * info.input_elems + off + e];
      check_cuda(cudaMemcpy(d_msg, m.data(), m.size() * 8, cudaMemcpyHostToDevice), "copy");
      check(pnb_encrypt_lwe(keys, d_msg, 1ull << scale, seed + 1, (uint64_t)off * batch, d_tmp,
                            (int)m.size(), nullptr),
            "encrypt");
      check_cuda(cudaMemcpy2D(d_in + off * L, (size_t)info.input_elems * L * 8, d_tmp,
                              (size_t)elems * L * 8, (size_t)elems * L * 8, batch,
                              cudaMemcpyDeviceToDevice),
                 "copy");
      off += elems;
    }
    check(pnb_evaluate(ev, d_in, batch, d_out, nullptr), "evaluate");
    check(pnb_phase_lwe(keys, d_out, d_ph, batch * (int)info.output_elems, 0, nullptr), "phase");
    std::vector<uint64_t> ph((size_t)batch * info.output_elems);
    check_cuda(cudaMemcpy(ph.data(), d_ph, ph.size() * 8, cudaMemcpyDeviceToHost), "copy");
    off = 0;
    for (int t = 0; t < info.num_outputs; ++t) {
      int64_t elems = 0;
      int scale = 0;
      check(pnb_plan_tensor(plan, 1, t, &elems, &scale, nullptr, nullptr), "output tensor");
      for (int b = 0; b < batch; ++b)
        for (int64_t e = 0; e < elems; ++e) {
          const uint64_t v = ph[(size_t)b * info.output_elems + off + e];
          y[(size_t)b * info.output_elems + off + e] =
              (int64_t)(v + (1ull << (scale - 1))) >> scale;
        }
      off += elems;
    }
    int status = 0;
    check(pnb_device_status(device, &status), "device status");
    if (status) die("a bounded device wait ran out (status " + std::to_string(status) + ")");
    cudaFree(d_in);
    cudaFree(d_out);
    cudaFree(d_msg);
    cudaFree(d_tmp);
    cudaFree(d_ph);
    pnb_evaluator_free(ev);
  }
  printf("{\"outputs\": [");
  for (int b = 0; b < batch; ++b) {
    printf("%s[", b ? ", " : "");
    for (int64_t e = 0; e < info.output_elems; ++e)
      printf("%s%lld", e ? ", " : "", (long long)y[(size_t)b * info.output_elems + e]);
    printf("]");
  }
  printf("]}\n");
  pnb_plan_free(plan);
  pnb_graph_free(graph);
  return 0;
}
