// ir.hpp -- the IR graph (model.fhe) as the reference defines it, with its load-time validation
// and bit-width budget.
//
// Mirrors runtime/src/ir.rs (Graph / Node / OpSpec, SCHEMA_VERSION "0.6.0", Graph::from_json
// at :169-180, OpSpec::build's checks at :197-452) and the bit-width growth rules and budget of
// runtime/src/eval.rs:182-276 with the per-op rules of runtime/src/ops/*.rs.  Error texts follow
// the reference's so that a caller sees the same diagnosis.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "json.hpp"

namespace pnb {
namespace ir {

constexpr const char* SCHEMA_VERSION = "0.6.0";
constexpr int MESSAGE_BITS = 2;

enum class OpType { Linear, Conv2d, Activation, Argmax, Requant, Pool, Add };

struct OpSpec {
  OpType type = OpType::Linear;
  // Linear / Conv2d
  std::vector<std::vector<int64_t>> weights;
  std::vector<int64_t> bias;
  int weight_bits = 0;
  int in_h = 0, in_w = 0, in_channels = 0, kernel_h = 0, kernel_w = 0, stride = 0, padding = 0;
  // Activation
  std::vector<uint64_t> lut;
  int output_bits = 0;
  // Argmax
  int64_t threshold = 0;
  // Requant
  uint32_t shift = 0;
  uint64_t mult = 1, round_bias = 0;
  int out_bits = 0;
  std::vector<uint64_t> clamp_lut;
  std::vector<uint64_t> mults, round_biases;
  std::vector<uint32_t> shifts;
  int channel_size = 0;  // 0 = per-tensor
  // Pool
  bool pool_avg = true;
  int channels = 0, pool_h = 0, pool_w = 0;

  const char* name() const;
};

struct Node {
  std::string name;
  std::vector<std::string> inputs, outputs;
  OpSpec op;
};

struct Graph {
  std::string schema_version;
  int num_blocks = 0;
  int input_bits = 0;
  std::vector<std::string> inputs, outputs;
  std::vector<Node> nodes;
};

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Parse + schema-version gate (Graph::from_json) and per-op validation (OpSpec::build).
Graph parse_graph(const char* json, size_t len);
void validate_op(const OpSpec& op);

// Bit-width propagation (eval.rs propagate_bit_widths) and the budget check
// (eval.rs check_graph_bit_width_budget).
std::unordered_map<std::string, int> propagate_bit_widths(const Graph& g);
void check_graph_bit_width_budget(const Graph& g);

// Output and internal bit widths of one op payload (JSON object) given its input widths: the
// per-op rules of Op::output_bits_n / Op::internal_bits_n (runtime/src/ops/mod.rs:77-138),
// after the op's validation.
void op_bits(const char* op_json, size_t len, const std::vector<int>& in_bits, int* output_bits,
             int* internal_bits);

// Flat output length of an op given its input lengths (the shape rule each op's eval asserts).
int64_t output_length(const OpSpec& op, const std::vector<int64_t>& in_lens);

}  // namespace ir
}  // namespace pnb
