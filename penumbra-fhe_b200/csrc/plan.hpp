// plan.hpp -- compile an IR graph into a batched ciphertext program.
//
// The reference walks the graph one sample at a time and evaluates every op with carry-
// propagating radix arithmetic (runtime/src/eval.rs:86-166, ops/*.rs).  Here every tensor
// element is ONE LWE ciphertext under the big key holding the exact integer value v at a
// power-of-two scale 2^e (phase = v * 2^e + noise, mod 2^64), and the graph becomes a straight
// program over whole batches:
//
//   Contract  Linear / Conv2d / avg-Pool: int8 weights x ciphertexts on the tensor cores
//   Lin       element-wise integer combinations (bias, thresholds, window corrections, Add)
//   Pbs       keyswitch + blind rotation + sample extraction with a per-element test vector
//
// Requant (runtime/src/ops/requant.rs:126-241), Activation (activation.rs:54-124) and Argmax
// (argmax.rs:22-35) become "threshold nodes".  Requant's
//     clamp_lut[ min((max(y,0)*mult + rb) >> shift, 2^out_bits - 1) ]
// equals clamp_lut[c0] + sum_j delta_j * [y >= T_j] over at most three integer thresholds
// T_j = ceil((j*2^shift - rb)/mult), j = c0+1 .. 2^out_bits-1, c0 = min(rb >> shift, max),
// delta_j = clamp_lut[j] - clamp_lut[j-1]; the indicators are nested, so the sum telescopes.
// Each [y >= T] is decided exactly by an LSB-first digit chain on v = y - T: windows of up to
// five bits are removed with two bootstraps each (one reads the window's top bit through the
// negacyclic sign, one reads the remaining bits with a lookup table), until v >> k fits a final
// sign bootstrap that emits delta_j * [v >= 0] at the output scale.  When the multiplier noise
// allows it the chain runs on z = mult*y + rb instead (the thresholds are then the aligned
// multiples of 2^shift, so all of them share the removal of the low `shift` bits).
//
// The planner tracks exact per-element value ranges (interval arithmetic), picks each tensor's
// scale from the ranges its consumers must represent, and picks for every bootstrap the
// cheapest key set (gadget base / levels) whose output noise keeps every later read within a
// z-sigma margin of its decision boundary.  `simulate` executes a program on noise-free phases,
// so the whole construction is checked on the CPU against the integer semantics.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "ir.hpp"

namespace pnb {
namespace plan {

struct KeyLevel {
  int base_log = 23, level = 1;
  double log2_sigma = 49.2;  // output noise std of one bootstrap (torus units, log2)
  double cost = 1.0;         // relative time of one bootstrap
};

// What the caller knows about one graph input when it is not a fresh client encryption (the
// output of an earlier op, evaluated one op at a time).
struct InputSpec {
  int scale = 0;          // plaintext scale (log2) the ciphertexts carry; 0 = the planner's choice
  double log2_sigma = 0;  // noise std (log2, torus units); 0 = a fresh encryption
  bool ranged = false;    // lo/hi below bound the values (otherwise input_lo / input_hi)
  int64_t lo = 0, hi = 0;
};

struct Options {
  int64_t input_lo = 0, input_hi = 0;  // declared range of every graph-input element
  std::vector<InputSpec> input_specs;  // per graph input (absent entries: defaults)
  int output_scale = 0;                // scale (log2) of every graph output; 0 = planner's choice
  double output_log2_sigma = 0;        // noise bound (log2 std) of every graph output; 0 = none
  bool check_budget = true;            // the reference's radix bit-width budget (whole graphs)
  double z = 7.0;                      // decision margin in standard deviations
  int n = 834, N = 2048;
  double log2_ksms = 54.83;   // keyswitch + modulus-switch noise std at the rotation input
  double log2_fresh = 15.68;  // client encryption noise std under the big key
  std::vector<KeyLevel> levels;  // available bootstrap key sets (any order)
  std::vector<int64_t> input_lens;  // per graph input (0 / absent: inferred from consumers)
};

struct Term {
  int src = -1;
  std::vector<int64_t> coef;  // per destination element, or one value for all
  std::vector<int32_t> map;   // source element per destination element (-1 skips); empty = same
};

struct TvSpec {  // test vector: lut_len boxes over the half torus, negacyclic continuation
  int lut_len = 1;
  std::vector<uint64_t> val;
};

enum class Kind { Contract, Lin, Pbs };

struct Instr {
  Kind kind = Kind::Lin;
  int dst = -1;
  // Lin: dst[e] = sum_t coef_t[e] * src_t[map_t[e]] + cst[e] (cst added to the body)
  std::vector<Term> terms;
  std::vector<uint64_t> cst;
  // Pbs: dst[e] = PBS_level(2^shift * src[e] + offset; tvs[tv[e]])
  int src = -1, shift = 0, level = 0;
  uint64_t offset = 0;
  std::vector<int32_t> tv;
  // Contract: dst[m*P + p] = sum_k W[m][k] * src[gather[p][k]] + bias[m] * bias_delta
  int M = 0, K = 0, P = 1;
  std::vector<int8_t> W;
  std::vector<int64_t> bias;
  uint64_t bias_delta = 0;
  std::vector<int32_t> gather;  // [P][K]; -1 = zero tap; empty = dense (P = 1, src = K elems)
  std::string what;
};

struct Buffer {
  int64_t elems = 0;
  std::string name;
};

struct TensorIO {
  std::string name;
  int buf = -1;
  int64_t elems = 0;
  int scale = 0;  // log2 of the plaintext scale
  double log2_sigma = 0;
  int64_t lo = 0, hi = 0;
};

struct Program {
  std::vector<Buffer> bufs;
  std::vector<TvSpec> tvs;
  std::vector<Instr> code;
  std::vector<KeyLevel> levels;  // key sets the program uses (Instr::level indexes this)
  std::vector<TensorIO> inputs, outputs;
  int64_t input_elems = 0, output_elems = 0;  // per sample, all tensors concatenated
  int64_t pbs_per_sample = 0;
  double cost_per_sample = 0;
  std::vector<int64_t> pbs_per_level;  // bootstraps per sample by key set (indexes levels)
  std::string report;
  Options opt;
};

// Throws ir::Error (message = the diagnosis) when the graph is invalid, exceeds the reference's
// bit-width budget, uses an op this path does not implement, or no exact plan exists.
Program build(const ir::Graph& g, const Options& o);

// Radix conversion programs between wide ciphertexts and the reference's radix blocks (one
// block per msg_bits digit of the integer, two's complement when is_signed, at the block scale
// 2^(63 - msg_bits - carry_bits); block 0 least significant).
//   split (to_blocks): input `wide` (elems integers at wide.scale with wide.log2_sigma noise,
//          values in [wide.lo, wide.hi]); output elems * num_blocks clean blocks, element-major.
//   merge: input elems * num_blocks blocks (digits up to block_max: clean, or with carries up
//          to the block space; fresh or bootstrapped); output elems integers at wide.scale (0: the widest that holds them)
//          with noise below wide.log2_sigma (0: decodable with the margin).
struct RadixSpec {
  bool to_blocks = true;
  bool is_signed = true;
  int num_blocks = 1;
  int msg_bits = 2, carry_bits = 2;
  int block_max = 0;  // merge: largest digit a block may hold (0: clean, 2^msg_bits - 1)
  int64_t elems = 1;
  InputSpec wide;
};
Program build_radix(const RadixSpec& r, const Options& o);

// Noise-free execution: inputs [batch][input_elems] integers, outputs [batch][output_elems]
// decoded integers.  min_margin receives the smallest distance (in units of 2^64/2N) between a
// bootstrap's exact input phase and the nearest boundary where its test vector changes value.
void simulate(const Program& prog, const int64_t* inputs, int batch, int64_t* outputs,
              double* min_margin);

// The N test-vector coefficients of a spec (what the blind rotation starts from).
std::vector<uint64_t> materialize_tv(const TvSpec& s, int N);

// Default key-set menu for a parameter set: output noise from the measured (default set) or
// analytic estimate, cost relative to the single-level key.
std::vector<KeyLevel> default_levels(int n, int N, int k, double glwe_std);
double ksms_log2_sigma(int n, int N, int k, int ks_base_log, int ks_level, double lwe_std);

}  // namespace plan
}  // namespace pnb
