/*
 * penumbra_b200.h -- C ABI of the B200 encrypted-evaluation library.
 *
 * The reference (Penumbra-FHE) evaluates an IR op graph on the CPU through the tfhe 1.6.3
 * crate; it has no FFI of its own.  Each entry point below replaces one tfhe-rs call family the
 * reference makes, so that an FFI shell over the reference runtime (a Rust `extern "C"` block,
 * a ctypes stub) can route the same operations here.  Conventions:
 *   - every function returns an int status (PNB_OK = 0); pnb_last_error() describes a failure;
 *   - pointers named *_dev are device (HBM) pointers on the key set's device, *_host are host;
 *   - ciphertexts are u64 words mod 2^64: an LWE ciphertext of dimension d is d+1 words with
 *     the body last; batches are contiguous [count][d+1];
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); calls are asynchronous on it
 *     unless documented otherwise and are thread-compatible (one stream per caller thread);
 *   - key sets and the per-device FFT tables the library builds at the first key set on a
 *     device live in that device's primary context: a cudaDeviceReset invalidates them, and
 *     the library must not be used on that device again in the same process.
 */
#ifndef PENUMBRA_B200_H
#define PENUMBRA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PNB_OK 0
#define PNB_ERR_INVALID 1     /* bad argument / shape / parameter */
#define PNB_ERR_CUDA 2        /* a CUDA runtime call failed */
#define PNB_ERR_OOM 3         /* device allocation failed */
#define PNB_ERR_TIMEOUT 4     /* a bounded device wait ran out */
#define PNB_ERR_UNSUPPORTED 5 /* parameters outside the compiled kernel set */

/* TFHE parameter set.  Field meaning follows tfhe-rs ClassicPBSParameters, which the reference
 * pins as DEFAULT_PARAMS = PARAM_MESSAGE_2_CARRY_2_KS_PBS (runtime/src/keys.rs:29). */
typedef struct pnb_params {
  int32_t n;            /* small LWE dimension (keyswitch output / blind-rotation input) */
  int32_t k;            /* GLWE dimension */
  int32_t N;            /* polynomial size */
  int32_t pbs_base_log; /* bootstrapping gadget: base 2^pbs_base_log ... */
  int32_t pbs_level;    /* ... with pbs_level levels */
  int32_t ks_base_log;  /* keyswitch gadget: base 2^ks_base_log ... */
  int32_t ks_level;     /* ... with ks_level levels */
  int32_t msg_bits;     /* message bits per block (reference MESSAGE_BITS = 2, keys.rs:36) */
  int32_t carry_bits;   /* carry bits per block */
  int32_t reserved;
  double lwe_std;       /* small-key noise std as a fraction of the torus */
  double glwe_std;      /* GLWE / big-key noise std as a fraction of the torus */
} pnb_params;

/* Opaque key set resident on one GPU: Fourier-domain bootstrapping key, keyswitching key and,
 * for the client-side harness, the secret keys. */
typedef struct pnb_keys pnb_keys;

/* Library version (major*10000 + minor*100 + patch) and the last error of the calling thread. */
int pnb_version(void);
const char* pnb_last_error(void);

/* Fill `out` with the library's default set: the Gaussian variant of
 * PARAM_MESSAGE_2_CARRY_2_KS_PBS (n=834, k=1, N=2048, PBS 2^23 x 1, KS 2^3 x 5).
 * Replaces: keys::DEFAULT_PARAMS (runtime/src/keys.rs:29). */
int pnb_params_default(pnb_params* out);

/* Fill `out` with the library's 6-bit set at N = 8192: n=1024, k=1, N=8192, PBS 2^23 x 1 (2^15 x 2
 * for low-noise bootstraps), KS 2^4 x 5, 3 message + 3 carry bits, small-key noise 2^-25, GLWE
 * noise 2^-62 (fractions of the torus).  The reference names a 6-bit N=8192 set only in its
 * benchmark configuration; these values are this library's choice (keyswitch + modulus-switch
 * noise about 2^52.8 and single-level bootstrap noise about 2^50.5 against a 2^57 message scale).
 * No reference counterpart (the reference's only set is keys::DEFAULT_PARAMS,
 * runtime/src/keys.rs:29). */
int pnb_params_n8192(pnb_params* out);

/* Generate secret keys, the bootstrapping key (then its Fourier form) and the keyswitching key
 * on `device` from `seed`; blocks until the keys are resident.
 * Replaces: keys::keygen -> tfhe gen_keys_radix (runtime/src/keys.rs:47-56). */
int pnb_keygen(int device, const pnb_params* params, uint64_t seed, pnb_keys** out);
/* Build a key set on `device` from key material on the host, in pnb_keys_export's layouts:
 * bsk (standard domain) and ksk are required; lwe_sk and glwe_sk are both given or both NULL.
 * Without them the set is an evaluation-key set (the server's view): bootstraps, keyswitches
 * and graph evaluation work, encryption and phases are refused.  The Fourier bootstrapping key
 * is computed on the device.  Blocking.  Replaces: deserialising a ServerKey / uploading the
 * client's evaluation keys (the keys the reference's keys::keygen returns, keys.rs:47-56). */
int pnb_keys_import(int device, const pnb_params* params, const uint64_t* lwe_sk_host,
                    const uint64_t* glwe_sk_host, const uint64_t* bsk_host,
                    const uint64_t* ksk_host, pnb_keys** out);
int pnb_keys_free(pnb_keys* keys);
int pnb_keys_info(const pnb_keys* keys, pnb_params* params_out, int* device_out,
                  size_t* fourier_bsk_bytes, size_t* ksk_bytes);
/* Copy key material to host buffers (any pointer may be NULL): lwe_sk[n], glwe_sk[k*N],
 * bsk[n*(k+1)*pbs_level*(k+1)*N] (standard domain), ksk[k*N*ks_level*(n+1)].  Blocking. */
int pnb_keys_export(const pnb_keys* keys, uint64_t* lwe_sk_host, uint64_t* glwe_sk_host,
                    uint64_t* bsk_host, uint64_t* ksk_host);

/* Byte containers (little-endian, versioned, self-describing) for shipping keys and ciphertexts
 * between a client and a GPU server.  A key set serialises its parameters, its standard-domain
 * bootstrapping key and keyswitching key (pnb_keys_export's layouts) and, with with_secrets,
 * the secret keys; deserialising computes the Fourier key on `device` (without secrets: an
 * evaluation-key set).  Ciphertext batches are [count][dim+1] u64 rows (mask, then body) in host
 * memory; pnb_lwe_deserialize with ct_host = NULL returns count and dim only.  The reference
 * serialises nothing (keys.rs:47-56 generates them in-process); tfhe-rs's own serialized format
 * cannot be checked here (the crate is absent), so these containers are this library's own. */
size_t pnb_keys_serialized_bytes(const pnb_keys* keys, int with_secrets);
int pnb_keys_serialize(const pnb_keys* keys, int with_secrets, void* out_host, size_t cap);
int pnb_keys_deserialize(int device, const void* in_host, size_t len, pnb_keys** out);
size_t pnb_lwe_serialized_bytes(int count, int dim);
int pnb_lwe_serialize(const uint64_t* ct_host, int count, int dim, void* out_host, size_t cap);
int pnb_lwe_deserialize(const void* in_host, size_t len, uint64_t* ct_host, size_t cap_words,
                        int* count, int* dim);

/* Client side (test harness).  Encrypt messages[i]*delta under the big (k*N) key with GLWE
 * noise; ciphertext i uses keystream index first_index+i of `seed`.
 * Replaces: encrypt::encrypt -> RadixClientKey::encrypt_signed (runtime/src/encrypt.rs:20-22). */
int pnb_encrypt_lwe(const pnb_keys* keys, const int64_t* messages_dev, uint64_t delta,
                    uint64_t seed, uint64_t first_index, uint64_t* ct_dev, int count,
                    void* stream);
/* Phase b - <a, s> of each ciphertext under the big key (small_key = 0) or small key (1).
 * Replaces the phase step of encrypt::decrypt_vec (runtime/src/encrypt.rs:43-45). */
int pnb_phase_lwe(const pnb_keys* keys, const uint64_t* ct_dev, uint64_t* phase_dev, int count,
                  int small_key, void* stream);

/* Build the blind-rotation test vector (N words) of a lookup table: box m of width N/lut_len
 * holds lut[m]*delta_out, rotated by half a box.
 * Replaces: ServerKey::generate_lookup_table (runtime/src/ops/activation.rs:104,
 * runtime/src/ops/requant.rs:193). */
int pnb_test_vector(const pnb_keys* keys, const uint64_t* lut_host, int lut_len,
                    uint64_t delta_out, uint64_t* tv_dev, void* stream);

/* Keyswitch a batch of big-key LWE ciphertexts [count][k*N+1] to the small key [count][n+1],
 * on the tensor cores.  `workspace` (>= pnb_keyswitch_workspace_bytes, 256-byte aligned) may be
 * NULL, in which case the digit scratch comes from the stream-ordered allocator.
 * Replaces: the keyswitch inside shortint apply_lookup_table (KS_PBS order,
 * runtime/src/ops/activation.rs:115). */
size_t pnb_keyswitch_workspace_bytes(const pnb_keys* keys, int count);
int pnb_keyswitch(const pnb_keys* keys, const uint64_t* in_dev, uint64_t* out_dev, int count,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Blind rotation + sample extraction of small-key ciphertexts [count][n+1] into big-key
 * ciphertexts [count][k*N+1] (the second half of pnb_pbs_batch, without the keyswitch).
 * Replaces: the programmable bootstrap inside shortint apply_lookup_table
 * (runtime/src/ops/activation.rs:115). */
int pnb_blind_rotate(const pnb_keys* keys, const uint64_t* tv_dev, const uint64_t* small_dev,
                     uint64_t* out_dev, int count, void* stream);

/* Bytes of device scratch pnb_pbs_batch needs for `count` ciphertexts. */
size_t pnb_pbs_workspace_bytes(const pnb_keys* keys, int count);

/* Programmable bootstrap of a batch: keyswitch, modulus switch, blind rotation with the
 * Fourier bootstrapping key, sample extraction.  in/out are [count][k*N+1] (may not alias).
 * `workspace` (>= pnb_pbs_workspace_bytes) may be NULL, in which case the scratch is taken
 * from the stream-ordered allocator for the duration of the call.
 * Replaces: shortint ServerKey::apply_lookup_table (runtime/src/ops/activation.rs:115,
 * runtime/src/ops/requant.rs:232), called once per ciphertext by the reference. */
int pnb_pbs_batch(const pnb_keys* keys, const uint64_t* tv_dev, const uint64_t* in_dev,
                  uint64_t* out_dev, int count, void* workspace, size_t workspace_bytes,
                  void* stream);

/* pnb_pbs_batch without any device allocation, for callers that cannot allocate GPU memory on
 * this path (memory already reserved by another framework's caching allocator, request loops
 * that must not pay allocator latency or synchronisation, FFI callers that keep a fixed device
 * footprint after start-up).  The scratch is a fixed 4 MiB array that every GPU loading the
 * library holds until exit; with the default parameter set a call takes at most 247
 * ciphertexts and larger counts are rejected with PNB_ERR_INVALID (split the batch).  Every
 * call looks up that array's device address on the current device (a lookup that allocates
 * nothing); make the first call on a device before any stream capture.  Calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.  The key set must
 * come from pnb_keygen or pnb_keys_import on the same device.
 * No counterpart in the reference. */
int pnb_pbs_batch_noalloc(const pnb_keys* keys, const uint64_t* tv_dev, const uint64_t* in_dev,
                          uint64_t* out_dev, int count, void* stream);

/* Merge radix integers into wide ciphertexts.  blocks_dev is [count][num_blocks][k*N+1]: one
 * integer per row, block 0 least significant, each block a big-key ciphertext of one digit
 * (msg_bits bits plus carries, delta 2^(63 - msg_bits - carry_bits)), as the reference encrypts
 * a signed radix integer.  out_dev [count][k*N+1] receives each integer v as v * delta_out
 * (mod 2^64).  With is_signed the top block's digit is read as two's complement and carries
 * above it are dropped; the result equals decrypt_signed's whenever the lower blocks' weighted
 * sum stays below the top block's weight, which holds for carry-free lower blocks (as
 * encrypt_signed and every carry-propagating radix op leave them).  Costs one bootstrap per
 * block plus one sum, with `keys`' gadget: the noise is the sum of num_blocks bootstrap
 * outputs of that key set, so decryption needs delta_out well above it (a multi-level key set
 * from the same seed merges wider integers) and |v| * delta_out < 2^62.  Requires
 * num_blocks * msg_bits <= 63 and num_blocks * 2^(msg_bits + carry_bits) <= 1024.  Allocates
 * its scratch from the stream-ordered allocator and does not synchronise the stream.
 * Replaces: RadixClientKey::encrypt_signed / decrypt_signed's block encoding at a graph
 * boundary (runtime/src/encrypt.rs:20-22, 43-45): ciphertexts in the reference's radix form
 * enter the wide-ciphertext kernels. */
int pnb_radix_merge(const pnb_keys* keys, const uint64_t* blocks_dev, int num_blocks, int count,
                    int is_signed, uint64_t delta_out, uint64_t* out_dev, void* stream);

/* Ciphertext x cleartext-weight contraction over LWE vectors mod 2^64, on the tensor cores:
 *   Y[b][j][c] = sum_i W[j][i] * X[b][i][c]  + (c == lwe_len-1 ? bias[j]*delta : 0)
 * W is int8 row-major [M][K] (K <= 65536), bias int64 [M] (may be NULL), X [batch][K][lwe_len],
 * Y [batch][M][lwe_len].  Runs on the current device.
 * Replaces: the per-row scalar_mul_parallelized / add_parallelized / scalar_add_parallelized
 * loops of Linear::eval (runtime/src/ops/linear.rs:52-75). */
int pnb_lwe_contract(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta, int M, int K,
                     const uint64_t* X_dev, uint64_t* Y_dev, int batch, int lwe_len,
                     void* stream);

/* Gathered contraction: Y[g][j][c] = sum_k W[j][k] * X[index[g][k]][c] (+ bias on the body),
 * index int32 [groups][K] selecting ciphertexts of X ([*][lwe_len]), -1 = a zero ciphertext.
 * An implicit im2col: one group per (sample, output position) of a convolution, or per pooling
 * window with W = 1.  Runs on the current device.
 * Replaces: Conv2d::eval's tap loops (runtime/src/ops/conv2d.rs:91-139) and the avg window sums
 * of Pool::eval (runtime/src/ops/pool.rs:110-118). */
int pnb_lwe_contract_gather(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta, int M,
                            int K, const uint64_t* X_dev, const int32_t* index_dev, int groups,
                            uint64_t* Y_dev, int lwe_len, void* stream);

/* The two contractions over ciphertext rows at explicit pitches: row r of X starts at word
 * r * ldx, row r of Y at r * ldy (ldx, ldy >= lwe_len).  An even ldx with a 16-byte aligned X
 * (2050 words for N = 2048, the layout the graph evaluator keeps) lets the operand move as TMA
 * tiles (dense) or 16-byte copies (gathered); an odd pitch takes 8-byte copies.  Replaces the
 * same reference loops as pnb_lwe_contract / pnb_lwe_contract_gather. */
int pnb_lwe_contract_ld(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta, int M,
                        int K, const uint64_t* X_dev, int ldx, uint64_t* Y_dev, int ldy,
                        int batch, int lwe_len, void* stream);
int pnb_lwe_contract_gather_ld(const int8_t* W_dev, const int64_t* bias_dev, uint64_t delta,
                               int M, int K, const uint64_t* X_dev, int ldx,
                               const int32_t* index_dev, int groups, uint64_t* Y_dev, int ldy,
                               int lwe_len, void* stream);

/* Negacyclic products out[c] = a[c] * b[c] mod (X^N + 1) through the same f64 FFT the blind
 * rotation uses (a: small signed integers, |a| < 2^31; b: u64 torus), count polynomials.
 * Diagnostic entry point for the FFT's precision; no reference counterpart. */
int pnb_fft_negacyclic_mul(int device, int N, const int64_t* a_dev, const uint64_t* b_dev,
                           uint64_t* out_dev, int count, void* stream);

/* Read and clear the device status words of the kernels with bounded waits: 0 when no wait ran
 * out since the last read; otherwise 1-3 keyswitch (producer, MMA, epilogue), 17 blind
 * rotation, 33 contraction.  No reference counterpart. */
int pnb_device_status(int device, int* status_out);

/* Measure this device's FP64 FMA throughput (TFLOP/s) with a short register-only kernel; the
 * roofline denominator of the blind rotation.  No reference counterpart. */
int pnb_measure_fp64_peak(int device, double* tflops_out);

/* Run the kernels' bounded mbarrier wait against a barrier that is never completed, with a limit
 * of `polls` polls (1..2^24): *warps_gave_up_out receives the number of waiting warps (2) that
 * gave up and reported it instead of hanging; the context stays usable.  The timeout path of the
 * device-side failure detection, exercised without a fault.  No reference counterpart. */
int pnb_wait_probe(int device, unsigned polls, int* warps_gave_up_out);

/* ---- Graph evaluation ------------------------------------------------------------------
 * The IR graph (a model.fhe document), compiled into a batched ciphertext program and run on
 * one GPU.  Every tensor element is one big-key LWE ciphertext holding the exact integer at a
 * per-tensor power-of-two scale (pnb_plan_tensor); Requant, Activation and Argmax are exact
 * bootstrap programs whose decrypted outputs equal the reference's integer semantics. */
typedef struct pnb_graph pnb_graph;
typedef struct pnb_plan pnb_plan;
typedef struct pnb_evaluator pnb_evaluator;

typedef struct pnb_plan_summary {
  int64_t input_elems;     /* ciphertexts per sample over all graph inputs, in graph order */
  int64_t output_elems;    /* ciphertexts per sample over all graph outputs, in graph order */
  int32_t num_inputs, num_outputs;
  int64_t pbs_per_sample;  /* bootstraps one sample costs */
  double cost_per_sample;  /* the same in single-level bootstrap equivalents */
  int32_t num_instructions;
  int32_t reserved;
} pnb_plan_summary;

/* Parse and validate a graph document (the graph object itself, or a document holding it under
 * "graph").  Same schema gate and op validation as the reference, with its messages.
 * Replaces: Graph::from_json + OpSpec::build (runtime/src/ir.rs:169-180, 197-452). */
int pnb_graph_load(const char* json, size_t len, pnb_graph** out);
int pnb_graph_free(pnb_graph* graph);
int pnb_graph_info(const pnb_graph* graph, int* num_nodes, int* num_blocks, int* input_bits);

/* Bit-width budget of the graph against its num_blocks radix (PNB_ERR_INVALID + message when
 * exceeded).  Replaces: check_graph_bit_width_budget (runtime/src/eval.rs:237-276). */
int pnb_graph_check_budget(const pnb_graph* graph);

/* Output and internal bit widths of one op (its IR payload, a JSON object such as a node's
 * "op") consuming tensors of the given widths, after the op's validation (PNB_ERR_INVALID +
 * the reference's message when it fails).  Replaces: Op::output_bits_n / Op::internal_bits_n
 * (runtime/src/ops/mod.rs:116-138) with the per-op rules of ops/{linear,conv2d,pool,requant,
 * activation,argmax,add}.rs. */
int pnb_op_bits(const char* op_json, size_t len, const int* input_bits, int n_inputs,
                int* output_bits, int* internal_bits);

/* Compile a graph for a parameter set.  input_lens (may be NULL; one entry per graph input, 0 =
 * infer from the consumer) gives the element count of each graph input; input_lo/input_hi bound
 * every graph-input value; margin_sigmas (<= 0: 7) is the decision margin of every bootstrap in
 * noise standard deviations.  Fails when the graph exceeds the budget or no exact program
 * exists.  Replaces: the per-node op construction of evaluate_graph (runtime/src/eval.rs:94-133). */
int pnb_plan_create(const pnb_graph* graph, const pnb_params* params, const int64_t* input_lens,
                    int64_t input_lo, int64_t input_hi, double margin_sigmas, pnb_plan** out);
int pnb_plan_free(pnb_plan* plan);
int pnb_plan_info(const pnb_plan* plan, pnb_plan_summary* info);
/* Element count, plaintext scale (log2) and value range of input (is_output = 0) or output
 * tensor idx.  Encrypt inputs at 2^scale_log2; decode outputs by signed rounding at 2^scale_log2. */
int pnb_plan_tensor(const pnb_plan* plan, int is_output, int idx, int64_t* elems,
                    int* scale_log2, int64_t* lo, int64_t* hi);
/* Key sets (gadget base_log, levels) the program bootstraps with and the bootstraps per sample
 * of each; fills up to `cap` entries and returns the number of key sets (-1 on a bad argument). */
int pnb_plan_key_sets(const pnb_plan* plan, int cap, int* base_log, int* level, int64_t* count);
/* Human-readable program summary (bytes needed including the terminator). */
size_t pnb_plan_report(const pnb_plan* plan, char* buf, size_t cap);
/* Noise-free host execution of the program on cleartext integers: inputs [batch][input_elems],
 * outputs [batch][output_elems]; min_margin (may be NULL) receives the smallest distance, in
 * units of 2^64/2N, from a bootstrap input to a decision boundary.  No GPU needed. */
int pnb_plan_simulate(const pnb_plan* plan, const int64_t* inputs, int batch, int64_t* outputs,
                      double* min_margin);

/* Create the GPU evaluator of a plan: generates on `device` every bootstrapping key set the
 * program uses from `seed` (all share the secret keys and the keyswitching key) and uploads the
 * program tables.  max_bytes bounds the per-chunk ciphertext buffers (0: half the free memory).
 * Replaces: keys::keygen + EvalCtx (runtime/src/keys.rs:47-56, ops/mod.rs:64-69). */
int pnb_evaluator_create(const pnb_plan* plan, int device, uint64_t seed, size_t max_bytes,
                         pnb_evaluator** out);
int pnb_evaluator_free(pnb_evaluator* ev);
/* Allocate the per-chunk buffers for batches of up to `batch` samples now (otherwise the first
 * pnb_evaluate of a larger batch allocates them).  Blocking. */
int pnb_evaluator_reserve(pnb_evaluator* ev, int batch);
/* The evaluator's client key set (borrowed): encrypt inputs / decrypt outputs with it. */
int pnb_evaluator_keys(const pnb_evaluator* ev, pnb_keys** keys);
/* Evaluate `batch` samples: in_dev [batch][input_elems][kN+1], out_dev
 * [batch][output_elems][kN+1] ciphertexts, on the evaluator's device.
 * Replaces: evaluate_graph (runtime/src/eval.rs:86-166), batched over samples. */
int pnb_evaluate(pnb_evaluator* ev, const uint64_t* in_dev, int batch, uint64_t* out_dev,
                 void* stream);

/* ---- One op at a time --------------------------------------------------------------------
 * The same exact programs, compiled for a single IR op whose inputs arrive from earlier ops, so
 * that an FFI shell keeping the reference's node walk (runtime/src/eval.rs:104-153) can route
 * each node to the GPU: Linear / Conv2d / avg Pool to pnb_lwe_contract(_gather), everything
 * else to a one-op plan run on a key ring.  A tensor is described by pnb_tensor_desc; the
 * output descriptor of one op is the input descriptor of the next. */
typedef struct pnb_keyring pnb_keyring;

typedef struct pnb_tensor_desc {
  int64_t elems;      /* elements (ciphertexts) per sample */
  int64_t lo, hi;     /* every element's integer value lies in [lo, hi] */
  int32_t scale_log2; /* each element encrypts v * 2^scale_log2 (0 in an input: planner's choice) */
  int32_t reserved;
  double log2_sigma;  /* noise std of the elements, log2 of torus units (0: a fresh encryption) */
} pnb_tensor_desc;

/* Every key set the exact programs may bootstrap with (the planner's gadget menu for `params`),
 * generated on `device` from one seed: all share the secret keys and the keyswitching key, so
 * ciphertexts pass between them freely.  Blocking.
 * Replaces: keys::keygen + the ServerKey an EvalCtx borrows (runtime/src/keys.rs:47-56,
 * runtime/src/ops/mod.rs:64-69). */
int pnb_keyring_create(int device, const pnb_params* params, uint64_t seed, pnb_keyring** out);
int pnb_keyring_free(pnb_keyring* ring);
/* Key set `idx` of the ring (borrowed); set 0 is the client's: encrypt and decrypt with it. */
int pnb_keyring_keys(const pnb_keyring* ring, int idx, pnb_keys** keys);

/* Compile one IR op (its JSON payload, as in a node's "op") over n_inputs (1, or 2 for Add)
 * input tensors described by `in`; out_scale_log2 (0: the planner's choice) pins the output's
 * scale and out_log2_sigma (0: decryptable with the margin) bounds the output's noise, so that
 * the ops after it can read it exactly.  Fails with the reference's validation message, or when no exact program exists for
 * the inputs' noise and range.  The plan's input/output tensors are read back with
 * pnb_plan_tensor_desc.  Replaces: OpSpec::build + Op::eval for one node
 * (runtime/src/ir.rs:197-452, runtime/src/ops/mod.rs:77-138). */
int pnb_op_plan_create(const char* op_json, size_t len, const pnb_params* params,
                       const pnb_tensor_desc* in, int n_inputs, int out_scale_log2,
                       double out_log2_sigma, double margin_sigmas, pnb_plan** out);
int pnb_plan_tensor_desc(const pnb_plan* plan, int is_output, int idx, pnb_tensor_desc* desc);
/* Conversion programs between wide ciphertexts and the reference's radix blocks (one block per
 * msg_bits digit, two's complement when is_signed, block 0 least significant, each block a
 * big-key ciphertext of its digit at the block scale 2^(63 - msg_bits - carry_bits), laid out
 * [element][num_blocks]).  Run them with an evaluator like any plan.
 *   to_blocks = 1 (split): `wide` describes the input integers (elems, value range, scale,
 *     noise); the output holds elems * num_blocks clean blocks.  Four bootstraps per digit
 *     (three for the top one): the digits are peeled off LSB first, each window read through the
 *     negacyclic sign and a two-box lookup, with the key sets that keep every later read exact.
 *   to_blocks = 0 (merge): the input holds elems * num_blocks blocks whose digits reach at most
 *     block_max (0: clean blocks, digits below 2^msg_bits, as encrypt_signed and every
 *     carry-propagating radix op leave them; up to 2^(msg_bits + carry_bits) - 1 with carries,
 *     which widens the integer); `wide` requests the output: elems, scale (0: the widest that holds the
 *     integers) and a noise bound (log2_sigma; 0: decodable with the margin).  One bootstrap per
 *     block, with the cheapest key set whose summed outputs meet the bound, then a sum.
 * Replaces: RadixClientKey::encrypt_signed / decrypt_signed's block encoding at graph
 * boundaries (runtime/src/encrypt.rs:20-22, 43-45; SignedRadixCiphertext,
 * runtime/src/ops/mod.rs:58). */
int pnb_radix_plan_create(const pnb_params* params, int num_blocks, int is_signed, int to_blocks,
                          int block_max, const pnb_tensor_desc* wide, double margin_sigmas,
                          pnb_plan** out);
/* An evaluator of `plan` that borrows the ring's key sets (no key generation) on the ring's
 * device.  The ring must outlive the evaluator. */
int pnb_evaluator_create_with(const pnb_plan* plan, const pnb_keyring* ring, size_t max_bytes,
                              pnb_evaluator** out);

/* Requant parameters: per-tensor (channels = 1) or per-channel (element e uses channel
 * e / channel_size), as the IR's Requant op carries them. */
typedef struct pnb_requant_spec {
  int32_t channels;
  int32_t out_bits;            /* <= 2 (MESSAGE_BITS) */
  int64_t channel_size;
  const uint64_t* mult;        /* [channels], each >= 1 */
  const uint64_t* round_bias;  /* [channels] */
  const uint32_t* shift;       /* [channels] */
  const uint64_t* clamp_lut;   /* [2^out_bits]; NULL = identity */
} pnb_requant_spec;

/* clamp_lut[min((max(v,0) * mult + round_bias) >> shift, 2^out_bits - 1)] of every element of
 * `batch` samples: in_dev [batch][in->elems][kN+1] wide ciphertexts, out_dev
 * [batch][in->elems][kN+1] at scale out_scale_log2 with noise below out_log2_sigma (0: the
 * planner's choice, as in pnb_op_plan_create; *out_desc, if given, receives the output's
 * descriptor).  Exact: decrypted outputs equal the integer op.
 * Blocking (compiles the element-wise program, runs it, synchronises `stream`).
 * Replaces: Requant::eval (runtime/src/ops/requant.rs:126-241). */
int pnb_requant_batch(const pnb_keyring* ring, const pnb_requant_spec* spec,
                      const pnb_tensor_desc* in, const uint64_t* in_dev, int batch,
                      int out_scale_log2, double out_log2_sigma, uint64_t* out_dev,
                      pnb_tensor_desc* out_desc, void* stream);
/* [v >= threshold] of a single-element tensor per sample (out_dev [batch][1][kN+1]).
 * Blocking.  Replaces: Argmax::eval (runtime/src/ops/argmax.rs:22-35). */
int pnb_argmax_batch(const pnb_keyring* ring, int64_t threshold, const pnb_tensor_desc* in,
                     const uint64_t* in_dev, int batch, int out_scale_log2,
                     double out_log2_sigma, uint64_t* out_dev, pnb_tensor_desc* out_desc,
                     void* stream);
/* a + b element-wise (both tensors at the same scale; out_scale_log2 0 or that scale).
 * Blocking.  Replaces: Add::eval_n (runtime/src/ops/add.rs:37-58). */
int pnb_add_batch(const pnb_keyring* ring, const pnb_tensor_desc* a, const uint64_t* a_dev,
                  const pnb_tensor_desc* b, const uint64_t* b_dev, int batch, int out_scale_log2,
                  double out_log2_sigma, uint64_t* out_dev, pnb_tensor_desc* out_desc,
                  void* stream);

/* ---- sample sharding across GPUs (one process per GPU) -------------------------------------
 * A batch is split into contiguous shards, rank r holding rows [start, stop) as pnb_shard
 * computes (sizes differ by at most one); every GPU evaluates its shard with its own key replica
 * (keys generated from the same seed are identical), then pnb_allgather reassembles the output
 * rows on every rank.  NCCL is opened at run time (libnccl.so.2; a process that already loaded
 * NCCL shares that copy) -- PNB_ERR_UNSUPPORTED when it cannot be.  The reference evaluates one
 * sample in one process (runtime/src/eval.rs:86-166) and has no collective; this is the
 * exchange step batching across GPUs adds. */
typedef struct pnb_comm pnb_comm;
#define PNB_COMM_ID_BYTES 128
int pnb_shard(int64_t batch, int world, int rank, int64_t* start, int64_t* stop);
/* One rank draws the id and hands its 128 bytes to the others out of band. */
int pnb_comm_unique_id(void* id_out);
/* Collective over `world` ranks: every rank calls it with the same id (blocking). */
int pnb_comm_create(int device, int world, int rank, const void* id, pnb_comm** out);
int pnb_comm_free(pnb_comm* comm);
/* Tears the communicator down without waiting for peers (after a peer failed). */
int pnb_comm_abort(pnb_comm* comm);
int pnb_comm_info(const pnb_comm* comm, int* device, int* world, int* rank);
/* PNB_OK, or the asynchronous NCCL error a collective hit (e.g. a peer that left). */
int pnb_comm_status(const pnb_comm* comm);
/* local_dev [stop - start][row_words] (this rank's shard of `batch` rows) -> out_dev
 * [batch][row_words] on every rank, enqueued on `stream`: one ncclAllGather for equal shards,
 * one grouped ncclBroadcast per rank into place for ragged ones.  local_dev may alias
 * out_dev + start * row_words. */
int pnb_allgather(pnb_comm* comm, const uint64_t* local_dev, uint64_t* out_dev, int64_t batch,
                  int64_t row_words, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* PENUMBRA_B200_H */
