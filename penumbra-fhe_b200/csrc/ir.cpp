// ir.cpp -- IR parsing, validation and bit-width budget (see ir.hpp for the reference map).
#include "ir.hpp"

#include <algorithm>
#include <set>

namespace pnb {
namespace ir {

const char* OpSpec::name() const {
  switch (type) {
    case OpType::Linear: return "Linear";
    case OpType::Conv2d: return "Conv2d";
    case OpType::Activation: return "Activation";
    case OpType::Argmax: return "Argmax";
    case OpType::Requant: return "Requant";
    case OpType::Pool: return "Pool";
    case OpType::Add: return "Add";
  }
  return "?";
}

namespace {

using json::Value;

[[noreturn]] void bad(const std::string& m) { throw Error(m); }

const Value& field(const Value& o, const char* k, const std::string& ctx) {
  const Value* v = o.get(k);
  if (!v) bad("IR parse error: missing field `" + std::string(k) + "` in " + ctx);
  return *v;
}
int64_t as_i64(const Value& v, const char* k) {
  if (v.kind != Value::Int || v.i_unsigned_overflow)
    bad(std::string("IR parse error: field `") + k + "` must be an integer");
  return v.i;
}
uint64_t as_u64(const Value& v, const char* k) {
  if (v.kind != Value::Int) bad(std::string("IR parse error: field `") + k + "` must be an integer");
  if (v.i_unsigned_overflow) return v.u;
  if (v.i < 0) bad(std::string("IR parse error: field `") + k + "` must be non-negative");
  return (uint64_t)v.i;
}
int as_usize(const Value& v, const char* k) {
  const int64_t x = as_i64(v, k);
  if (x < 0 || x > INT32_MAX) bad(std::string("IR parse error: field `") + k + "` out of range");
  return (int)x;
}
std::vector<std::string> strings(const Value& v, const char* k) {
  if (v.kind != Value::Array) bad(std::string("IR parse error: `") + k + "` must be an array");
  std::vector<std::string> out;
  for (const auto& e : v.arr) {
    if (e.kind != Value::String) bad(std::string("IR parse error: `") + k + "` holds non-strings");
    out.push_back(e.s);
  }
  return out;
}
std::vector<int64_t> ints(const Value& v, const char* k) {
  if (v.kind != Value::Array) bad(std::string("IR parse error: `") + k + "` must be an array");
  std::vector<int64_t> out;
  for (const auto& e : v.arr) out.push_back(as_i64(e, k));
  return out;
}
std::vector<uint64_t> uints(const Value& v, const char* k) {
  if (v.kind != Value::Array) bad(std::string("IR parse error: `") + k + "` must be an array");
  std::vector<uint64_t> out;
  for (const auto& e : v.arr) out.push_back(as_u64(e, k));
  return out;
}
std::vector<std::vector<int64_t>> matrix(const Value& v, const char* k) {
  if (v.kind != Value::Array) bad(std::string("IR parse error: `") + k + "` must be an array");
  std::vector<std::vector<int64_t>> out;
  for (const auto& row : v.arr) out.push_back(ints(row, k));
  return out;
}

OpSpec parse_op(const Value& o) {
  if (o.kind != Value::Object) bad("IR parse error: `op` must be an object");
  const Value& t = field(o, "op_type", "op");
  if (t.kind != Value::String) bad("IR parse error: `op_type` must be a string");
  OpSpec op;
  const std::string& ty = t.s;
  if (ty == "Linear") {
    op.type = OpType::Linear;
    op.weights = matrix(field(o, "weights", ty), "weights");
    op.bias = ints(field(o, "bias", ty), "bias");
    op.weight_bits = as_usize(field(o, "weight_bits", ty), "weight_bits");
  } else if (ty == "Conv2d") {
    op.type = OpType::Conv2d;
    op.weights = matrix(field(o, "weights", ty), "weights");
    op.bias = ints(field(o, "bias", ty), "bias");
    op.weight_bits = as_usize(field(o, "weight_bits", ty), "weight_bits");
    op.in_h = as_usize(field(o, "in_h", ty), "in_h");
    op.in_w = as_usize(field(o, "in_w", ty), "in_w");
    op.in_channels = as_usize(field(o, "in_channels", ty), "in_channels");
    op.kernel_h = as_usize(field(o, "kernel_h", ty), "kernel_h");
    op.kernel_w = as_usize(field(o, "kernel_w", ty), "kernel_w");
    op.stride = as_usize(field(o, "stride", ty), "stride");
    op.padding = as_usize(field(o, "padding", ty), "padding");
  } else if (ty == "Activation") {
    op.type = OpType::Activation;
    op.lut = uints(field(o, "lut", ty), "lut");
    op.output_bits = as_usize(field(o, "output_bits", ty), "output_bits");
  } else if (ty == "Argmax") {
    op.type = OpType::Argmax;
    op.threshold = as_i64(field(o, "threshold", ty), "threshold");
  } else if (ty == "Requant") {
    op.type = OpType::Requant;
    const int64_t sh = as_i64(field(o, "shift", ty), "shift");
    if (sh < 0 || sh > UINT32_MAX) bad("IR parse error: `shift` out of range");
    op.shift = (uint32_t)sh;
    op.mult = o.get("mult") ? as_u64(*o.get("mult"), "mult") : 1;  // serde default 1
    op.round_bias = o.get("round_bias") ? as_u64(*o.get("round_bias"), "round_bias") : 0;
    op.out_bits = as_usize(field(o, "out_bits", ty), "out_bits");
    op.clamp_lut = uints(field(o, "clamp_lut", ty), "clamp_lut");
    if (o.get("mults")) op.mults = uints(*o.get("mults"), "mults");
    if (o.get("round_biases")) op.round_biases = uints(*o.get("round_biases"), "round_biases");
    if (o.get("shifts")) {
      for (uint64_t s : uints(*o.get("shifts"), "shifts")) op.shifts.push_back((uint32_t)s);
    }
    const Value* cs = o.get("channel_size");
    op.channel_size = (cs && cs->kind != Value::Null) ? std::max(0, as_usize(*cs, "channel_size"))
                                                       : -1;  // -1 = absent
  } else if (ty == "Pool") {
    op.type = OpType::Pool;
    const Value& m = field(o, "mode", ty);
    if (m.kind != Value::String) bad("IR parse error: `mode` must be a string");
    if (m.s == "avg") op.pool_avg = true;
    else if (m.s == "max") op.pool_avg = false;
    else bad("Pool mode must be \"avg\" or \"max\"; got \"" + m.s + "\"");
    op.in_h = as_usize(field(o, "in_h", ty), "in_h");
    op.in_w = as_usize(field(o, "in_w", ty), "in_w");
    op.channels = as_usize(field(o, "channels", ty), "channels");
    op.pool_h = as_usize(field(o, "pool_h", ty), "pool_h");
    op.pool_w = as_usize(field(o, "pool_w", ty), "pool_w");
    op.stride = as_usize(field(o, "stride", ty), "stride");
  } else if (ty == "Add") {
    op.type = OpType::Add;
  } else {
    bad("IR parse error: unknown variant `" + ty +
        "`, expected one of `Linear`, `Conv2d`, `Activation`, `Argmax`, `Requant`, `Pool`, `Add`");
  }
  return op;
}

int magnitude_bits(uint64_t x) { return x ? 64 - __builtin_clzll(x) : 0; }

int ceil_log2(int64_t n) {  // ceil(log2 n) for n >= 1; 0 for n <= 1
  if (n <= 1) return 0;
  return 64 - __builtin_clzll((uint64_t)(n - 1));
}

int lut_output_bits(const std::vector<uint64_t>& lut) {
  uint64_t m = 0;
  for (uint64_t v : lut) m = std::max(m, v);
  return std::max(1, magnitude_bits(m));
}

int accumulator_bits(const OpSpec& op, int input_bits, int64_t fan_in) {
  const int sum_bits = input_bits + op.weight_bits + ceil_log2(fan_in);
  uint64_t mb = 0;
  for (int64_t b : op.bias) mb = std::max(mb, (uint64_t)(b < 0 ? -(uint64_t)b : (uint64_t)b));
  return std::max(sum_bits, magnitude_bits(mb)) + 2;
}

// requant.rs requant_internal_bits (u128 arithmetic)
int requant_internal_bits(int input_bits, uint64_t mult, uint64_t rb) {
  unsigned __int128 relu_max = input_bits >= 1 ? (((unsigned __int128)1 << (input_bits - 1)) - 1)
                                               : 0;
  unsigned __int128 peak = relu_max * mult + rb;
  int mag = 0;
  while (peak) { ++mag; peak >>= 1; }
  return std::max(mag + 1, input_bits);
}

int op_output_bits(const OpSpec& op, const std::vector<int>& in_bits) {
  auto single = [&]() {
    if (in_bits.size() != 1) bad("this op is single-input; override eval_n for a multi-input op");
    return in_bits[0];
  };
  switch (op.type) {
    case OpType::Linear:
      return accumulator_bits(op, single(), op.weights.empty() ? 0 : op.weights[0].size());
    case OpType::Conv2d:
      return accumulator_bits(op, single(), (int64_t)op.in_channels * op.kernel_h * op.kernel_w);
    case OpType::Pool: {
      const int b = single();
      return op.pool_avg ? b + ceil_log2((int64_t)op.pool_h * op.pool_w) : b;
    }
    case OpType::Requant: {
      single();
      const int derived = lut_output_bits(op.clamp_lut);
      if (op.out_bits < derived)
        bad("Requant out_bits (" + std::to_string(op.out_bits) + ") is smaller than the "
            "clamp_lut's actual range (" + std::to_string(derived) + " bits)");
      if (op.out_bits > MESSAGE_BITS)
        bad("Requant out_bits (" + std::to_string(op.out_bits) + ") exceeds MESSAGE_BITS (2)");
      return op.out_bits;
    }
    case OpType::Activation: {
      const int b = single();
      if (b > MESSAGE_BITS)
        bad("Activation input is wider (" + std::to_string(b) + " bits) than the single 2-bit "
            "block it consumes; activations need a Requant in front to narrow the value first");
      const int derived = lut_output_bits(op.lut);
      if (op.output_bits < derived)
        bad("Activation output_bits (" + std::to_string(op.output_bits) + ") is smaller than the "
            "LUT's actual range (" + std::to_string(derived) + " bits)");
      if (op.output_bits > MESSAGE_BITS)
        bad("Activation output_bits (" + std::to_string(op.output_bits) +
            ") exceeds MESSAGE_BITS (2)");
      return op.output_bits;
    }
    case OpType::Argmax:
      single();
      return 1;
    case OpType::Add:
      if (in_bits.size() != 2)
        bad("Add takes exactly two inputs; got " + std::to_string(in_bits.size()));
      return std::max(in_bits[0], in_bits[1]) + 1;
  }
  return 0;
}

int op_internal_bits(const OpSpec& op, const std::vector<int>& in_bits) {
  if (op.type != OpType::Requant) return op_output_bits(op, in_bits);
  if (in_bits.size() != 1)
    bad("Requant is single-input; got " + std::to_string(in_bits.size()) + " input widths");
  if (op.mults.empty()) return requant_internal_bits(in_bits[0], op.mult, op.round_bias);
  int m = 0;
  for (size_t c = 0; c < op.mults.size(); ++c)
    m = std::max(m, requant_internal_bits(in_bits[0], op.mults[c], op.round_biases[c]));
  return m;
}

}  // namespace

void op_bits(const char* op_json, size_t len, const std::vector<int>& in_bits, int* output_bits,
             int* internal_bits) {
  Value v;
  try {
    v = json::parse(op_json, len);
  } catch (const std::exception& e) {
    bad(std::string("IR parse error: ") + e.what());
  }
  const OpSpec op = parse_op(v);
  validate_op(op);
  *output_bits = op_output_bits(op, in_bits);
  *internal_bits = op_internal_bits(op, in_bits);
}

void validate_op(const OpSpec& op) {
  switch (op.type) {
    case OpType::Linear: {
      if (op.weights.empty()) bad("Linear op has no weight rows");
      if (op.weights.size() != op.bias.size())
        bad("Linear op has " + std::to_string(op.weights.size()) + " weight rows but " +
            std::to_string(op.bias.size()) + " biases; need one bias per row");
      const size_t w = op.weights[0].size();
      for (size_t i = 0; i < op.weights.size(); ++i)
        if (op.weights[i].size() != w)
          bad("Linear weight row " + std::to_string(i) + " has width " +
              std::to_string(op.weights[i].size()) + " but row 0 has width " + std::to_string(w) +
              "; all rows must match the input length");
      break;
    }
    case OpType::Conv2d: {
      if (op.weights.empty()) bad("Conv2d op has no output channels (empty weights)");
      if (op.weights.size() != op.bias.size())
        bad("Conv2d has " + std::to_string(op.weights.size()) + " kernels but " +
            std::to_string(op.bias.size()) + " biases; need one bias per output channel");
      if (op.in_h == 0 || op.in_w == 0 || op.in_channels == 0)
        bad("Conv2d in_h/in_w/in_channels must be positive");
      if (op.kernel_h == 0 || op.kernel_w == 0 || op.stride == 0)
        bad("Conv2d kernel_h/kernel_w/stride must be positive");
      const size_t fan = (size_t)op.in_channels * op.kernel_h * op.kernel_w;
      for (size_t i = 0; i < op.weights.size(); ++i)
        if (op.weights[i].size() != fan)
          bad("Conv2d kernel row " + std::to_string(i) + " has width " +
              std::to_string(op.weights[i].size()) + " but in_channels*kernel_h*kernel_w = " +
              std::to_string(fan) + "; every kernel must match the fan-in");
      if (op.kernel_h > op.in_h + 2 * op.padding || op.kernel_w > op.in_w + 2 * op.padding)
        bad("Conv2d kernel (" + std::to_string(op.kernel_h) + "x" + std::to_string(op.kernel_w) +
            ") does not fit the padded input (" + std::to_string(op.in_h + 2 * op.padding) + "x" +
            std::to_string(op.in_w + 2 * op.padding) + ")");
      break;
    }
    case OpType::Requant: {
      const size_t domain = (size_t)1 << MESSAGE_BITS;
      if (op.clamp_lut.size() != domain)
        bad("Requant clamp_lut must have 4 entries (the 2-bit message space); got " +
            std::to_string(op.clamp_lut.size()));
      for (size_t i = 0; i < op.clamp_lut.size(); ++i)
        if (op.clamp_lut[i] >= domain)
          bad("Requant clamp_lut[" + std::to_string(i) + "] = " +
              std::to_string(op.clamp_lut[i]) + " does not fit one shortint block (must be < 4)");
      if (op.out_bits > MESSAGE_BITS)
        bad("Requant out_bits (" + std::to_string(op.out_bits) +
            ") exceeds MESSAGE_BITS (2); the narrowed value must fit a single shortint block");
      if (op.mult == 0) bad("Requant mult must be >= 1 (a fixed-point multiplier; 1 is a pure shift)");
      const bool has_pc = !op.mults.empty() || !op.shifts.empty() || !op.round_biases.empty() ||
                          op.channel_size >= 0;
      if (has_pc) {
        if (op.mults.empty())
          bad("Requant per-channel overlay present but `mults` is empty; supply one multiplier "
              "per output channel");
        if (op.shifts.size() != op.mults.size() || op.round_biases.size() != op.mults.size())
          bad("Requant per-channel arrays must be equal length: mults=" +
              std::to_string(op.mults.size()) + ", shifts=" + std::to_string(op.shifts.size()) +
              ", round_biases=" + std::to_string(op.round_biases.size()));
        if (op.channel_size < 0)
          bad("Requant per-channel overlay needs `channel_size` (elements per channel: 1 for a "
              "Linear head, out_h*out_w for a Conv2d)");
        if (op.channel_size < 1) bad("Requant channel_size must be >= 1");
        for (size_t i = 0; i < op.mults.size(); ++i)
          if (op.mults[i] == 0)
            bad("Requant mults[" + std::to_string(i) +
                "] = 0 must be >= 1 (a fixed-point multiplier per channel; 1 is a pure shift)");
      }
      break;
    }
    case OpType::Pool: {
      if (op.in_h == 0 || op.in_w == 0 || op.channels == 0)
        bad("Pool in_h/in_w/channels must be positive");
      if (op.pool_h == 0 || op.pool_w == 0 || op.stride == 0)
        bad("Pool pool_h/pool_w/stride must be positive");
      if (op.pool_h > op.in_h || op.pool_w > op.in_w)
        bad("Pool window (" + std::to_string(op.pool_h) + "x" + std::to_string(op.pool_w) +
            ") must fit the input (" + std::to_string(op.in_h) + "x" + std::to_string(op.in_w) +
            ")");
      break;
    }
    case OpType::Activation: {
      if (op.lut.size() != ((size_t)1 << MESSAGE_BITS))
        bad("Activation LUT must cover the full 2-bit message space (4 entries); got " +
            std::to_string(op.lut.size()));
      for (size_t i = 0; i < op.lut.size(); ++i)
        if (op.lut[i] >= 4)
          bad("Activation LUT entry lut[" + std::to_string(i) + "] = " +
              std::to_string(op.lut[i]) + " does not fit one shortint block");
      break;
    }
    default:
      break;
  }
}

Graph parse_graph(const char* text, size_t len) {
  json::Value root;
  try {
    root = json::parse(text, len);
  } catch (const std::exception& e) {
    bad(std::string("IR parse error: ") + e.what());
  }
  if (root.kind != Value::Object) bad("IR parse error: the graph must be a JSON object");
  // accept a fixture document that nests the graph under "graph"
  const Value* g = root.get("graph") ? root.get("graph") : &root;
  Graph G;
  const Value& sv = field(*g, "schema_version", "graph");
  if (sv.kind != Value::String) bad("IR parse error: `schema_version` must be a string");
  G.schema_version = sv.s;
  G.num_blocks = as_usize(field(*g, "num_blocks", "graph"), "num_blocks");
  G.input_bits = as_usize(field(*g, "input_bits", "graph"), "input_bits");
  G.inputs = strings(field(*g, "inputs", "graph"), "inputs");
  G.outputs = strings(field(*g, "outputs", "graph"), "outputs");
  const Value& nodes = field(*g, "nodes", "graph");
  if (nodes.kind != Value::Array) bad("IR parse error: `nodes` must be an array");
  for (const auto& n : nodes.arr) {
    Node node;
    const Value& nm = field(n, "name", "node");
    if (nm.kind != Value::String) bad("IR parse error: node `name` must be a string");
    node.name = nm.s;
    node.inputs = strings(field(n, "inputs", "node"), "inputs");
    node.outputs = strings(field(n, "outputs", "node"), "outputs");
    node.op = parse_op(field(n, "op", "node"));
    G.nodes.push_back(std::move(node));
  }
  if (G.schema_version != SCHEMA_VERSION)
    bad("IR schema-version mismatch: file declares \"" + G.schema_version +
        "\" but this runtime expects \"" + SCHEMA_VERSION +
        "\". A schema-version change is breaking; regenerate the IR from a matching front end.");
  return G;
}

std::unordered_map<std::string, int> propagate_bit_widths(const Graph& g) {
  std::unordered_map<std::string, int> w;
  for (const auto& name : g.inputs) w[name] = g.input_bits;
  for (const auto& node : g.nodes) {
    validate_op(node.op);
    if (node.inputs.empty() || node.outputs.size() != 1)
      bad("node '" + node.name + "' (" + node.op.name() +
          ") must have at least one input and exactly one output");
    std::vector<int> in;
    for (const auto& i : node.inputs) {
      auto it = w.find(i);
      if (it == w.end())
        bad("node '" + node.name + "' reads tensor '" + i +
            "', which no earlier node produced and is not a graph input — node order is not a "
            "valid topological order");
      in.push_back(it->second);
    }
    const int out = op_output_bits(node.op, in);
    if (w.count(node.outputs[0]))
      bad("node '" + node.name + "' writes tensor '" + node.outputs[0] +
          "', which already exists — tensor names must be unique");
    w[node.outputs[0]] = out;
  }
  return w;
}

void check_graph_bit_width_budget(const Graph& g) {
  const int capacity = g.num_blocks * MESSAGE_BITS;
  auto w = propagate_bit_widths(g);
  for (const auto& node : g.nodes) {
    const std::string& name = node.outputs[0];
    const int bits = w[name];
    if (bits > capacity)
      bad("bit-width budget exceeded at node '" + node.name + "' (tensor '" + name +
          "'): requires " + std::to_string(bits) + " bits but the radix holds only " +
          std::to_string(capacity) + " (" + std::to_string(g.num_blocks) +
          " blocks × 2 bits). Reduce precision or widen num_blocks (a Requant here is Phase 4).");
    std::vector<int> in;
    for (const auto& i : node.inputs) in.push_back(w[i]);
    const int internal = op_internal_bits(node.op, in);
    if (internal > capacity)
      bad("bit-width budget exceeded inside node '" + node.name + "' (" + node.op.name() +
          "): its rescale needs " + std::to_string(internal) +
          " transient bits (the multiply-then-shift intermediate) but the radix holds only " +
          std::to_string(capacity) + " (" + std::to_string(g.num_blocks) +
          " blocks × 2 bits). Reduce the requant multiplier, reduce input precision, or widen "
          "num_blocks.");
  }
}

int64_t output_length(const OpSpec& op, const std::vector<int64_t>& in_lens) {
  switch (op.type) {
    case OpType::Linear:
      if (in_lens[0] != (int64_t)op.weights[0].size())
        bad("Linear weight row width (" + std::to_string(op.weights[0].size()) +
            ") must match input length (" + std::to_string(in_lens[0]) + ")");
      return (int64_t)op.weights.size();
    case OpType::Conv2d: {
      if (in_lens[0] != (int64_t)op.in_channels * op.in_h * op.in_w)
        bad("Conv2d input length " + std::to_string(in_lens[0]) +
            " != in_channels*in_h*in_w = " + std::to_string(op.in_channels) + "*" +
            std::to_string(op.in_h) + "*" + std::to_string(op.in_w));
      const int oh = (op.in_h + 2 * op.padding - op.kernel_h) / op.stride + 1;
      const int ow = (op.in_w + 2 * op.padding - op.kernel_w) / op.stride + 1;
      return (int64_t)op.weights.size() * oh * ow;
    }
    case OpType::Pool: {
      if (in_lens[0] != (int64_t)op.channels * op.in_h * op.in_w)
        bad("Pool input length " + std::to_string(in_lens[0]) + " != channels*in_h*in_w = " +
            std::to_string(op.channels) + "*" + std::to_string(op.in_h) + "*" +
            std::to_string(op.in_w));
      const int oh = (op.in_h - op.pool_h) / op.stride + 1;
      const int ow = (op.in_w - op.pool_w) / op.stride + 1;
      return (int64_t)op.channels * oh * ow;
    }
    case OpType::Requant: {
      if (!op.mults.empty()) {
        if (in_lens[0] % op.channel_size != 0)
          bad("Requant per-channel: " + std::to_string(in_lens[0]) +
              " elements not divisible by channel_size " + std::to_string(op.channel_size));
        if (in_lens[0] / op.channel_size != (int64_t)op.mults.size())
          bad("Requant per-channel: " + std::to_string(in_lens[0] / op.channel_size) +
              " channels (len " + std::to_string(in_lens[0]) + " / channel_size " +
              std::to_string(op.channel_size) + ") != " + std::to_string(op.mults.size()) +
              " multipliers");
      }
      return in_lens[0];
    }
    case OpType::Activation:
      return in_lens[0];
    case OpType::Argmax:
      if (in_lens[0] != 1)
        bad("Argmax expects a single-logit input, got " + std::to_string(in_lens[0]) +
            " elements");
      return 1;
    case OpType::Add:
      if (in_lens.size() != 2 || in_lens[0] != in_lens[1])
        bad("Add operands must have equal length");
      return in_lens[0];
  }
  return 0;
}

}  // namespace ir
}  // namespace pnb
