/* bsml_decoder.h — C ABI of the B200-native Kokoro decoder training path.
 *
 * Drop-in boundary for the reference's decoder backward path
 * (wlejon/brosoundml: src/kokoro_decoder_backward.h, include/brosoundml/decoder_lora.h).
 * Every entry point takes plain device pointers and sizes; no C++ or torch type
 * crosses it. All functions return 0 on success, a negative status on failure;
 * bsml_last_error() gives the message ("brosoundml: <where>: <reason>", the
 * reference's error format, src/kokoro_modules.cpp:90-92).
 *
 * Layouts follow the reference: activations NCL, element (b, c, l) at
 * (b*C + c)*L + l (src/kokoro_decoder_backward.h:15-17, with a leading batch
 * axis); conv weights (C_out, C_in, k) (include/brosoundml/modules.h:75);
 * ConvTranspose1d weights (C_in, C_out, k) (include/brosoundml/kokoro_modules.h:321);
 * AdaIN affines (gamma, beta) each (C) per clip (src/kokoro_decoder_backward.h:37-56).
 * Streams are passed as void* (a cudaStream_t; NULL = legacy default stream).
 */
#ifndef BSML_DECODER_H
#define BSML_DECODER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Architecture. Field meanings follow DecoderBackbone::load_from
 * (src/kokoro_modules.cpp:1021-1063), Generator::load_from (:1237-1347) and
 * HarmonicSource::load_from (:1556-1572). */
typedef struct bsml_decoder_config {
    int asr_dim;          /* 512 */
    int style_dim;        /* 128 */
    int asr_res_dim;      /* 64 */
    int enc_dim;          /* 1024 */
    int n_decode;         /* 4 */
    int dec_out[8];       /* 1024, 1024, 1024, 512 */
    int upsample_block;   /* 3 */
    int n_ups;            /* 2 */
    int init_ch;          /* 512 */
    int ups_rate[4];      /* 10, 6 */
    int ups_kernel[4];    /* 20, 12 */
    int noise_kernel[4];  /* 12, 1 */
    int noise_stride[4];  /* 6, 1 */
    int noise_pad[4];     /* 3, 0 */
    int nr_kernel[4];     /* 7, 11 */
    int nr_dil[4][3];     /* {1,3,5} */
    int n_kernels;        /* 3 */
    int rb_kernel[4];     /* 3, 7, 11 */
    int rb_dil[4][3];     /* {1,3,5} */
    int har_ch;           /* 22 */
    int n_fft;            /* 20 */
    int hop;              /* 5 */
    int post_kernel;      /* 7 */
    int harmonic_num;     /* 8 */
    int sample_rate;      /* 24000 */
    int upsample_scale;   /* 300 */
} bsml_decoder_config;

typedef struct bsml_param_entry {
    char name[96];        /* upstream state-dict key below decoder.module. */
    int64_t offset;       /* in floats, into the flat parameter / gradient buffer */
    int64_t numel;
    int ndim;
    int shape[3];
    int trainable;
} bsml_param_entry;

typedef struct bsml_decoder bsml_decoder;

/* Arithmetic used for the conv / convT contractions. FP32_SIMT: fp32 CUDA-core
 * kernels. TF32X3: tcgen05 tensor cores, each fp32 operand split hi+lo, three
 * products (fp32-equivalent accuracy). BF16: tcgen05 with bf16 operands, fp32
 * accumulation. BF16X3: each operand split into bf16 hi + bf16 lo, three products
 * at the bf16 rate (about 16 bits of operand precision). TF32X3W: TF32X3 for the
 * forward and input-gradient contractions, BF16X3 for the weight gradients (their
 * rounding ends in dW and propagates nowhere; the whole gradient stays within the
 * TF32X3 bar at the benchmarked configuration). TF32X3F: TF32X3 for the forward
 * contractions only, BF16X3 for every contraction of the backward (input and weight
 * gradients): the decoder's gradients are sensitive to the forward's rounding, not
 * to the backward's, and stay within the TF32X3 bar. Elementwise, normalisation and
 * spectral work is fp32 in all modes. */
enum {
    BSML_MATH_FP32_SIMT = 0,
    BSML_MATH_TF32X3 = 1,
    BSML_MATH_BF16 = 2,
    BSML_MATH_BF16X3 = 3,
    BSML_MATH_TF32X3W = 4,
    BSML_MATH_TF32X3F = 5
};

const char* bsml_last_error(void);
int bsml_version(void);

/* ── whole-decoder engine ──────────────────────────────────────────────────
 * Replaces DecoderLora::forward / ::backward (src/decoder_lora.cpp:211-296)
 * and the assemblies they call (decoder_backbone_forward_train / _backward,
 * generator_forward_train / _backward, src/kokoro_decoder_backward.h:213-293),
 * batched over B clips. */
int bsml_decoder_create(const bsml_decoder_config* cfg, int device, bsml_decoder** out);
void bsml_decoder_destroy(bsml_decoder* d);
int bsml_decoder_param_count(const bsml_decoder* d, int64_t* n_params, int* n_entries, int* n_affine,
                             int64_t* aff_per_clip);
/* aff_channels (optional) receives the channel count of each AdaIN, in
 * DecoderLora::adapters() order (src/decoder_lora.cpp:173-179). */
int bsml_decoder_param_table(const bsml_decoder* d, bsml_param_entry* out, int max_entries, int* aff_channels);
int bsml_decoder_set_math(bsml_decoder* d, int math_mode);

/* The same layout queries from a config alone (no device needed). */
int bsml_config_param_count(const bsml_decoder_config* cfg, int64_t* n_params, int* n_entries, int* n_affine,
                            int64_t* aff_per_clip);
int bsml_config_param_table(const bsml_decoder_config* cfg, bsml_param_entry* out, int max_entries,
                            int* aff_channels);

/* Forward. params: flat (n_params). asr (B, asr_dim, T); F0, N (B, 2T);
 * style (B, style_dim); har (B, har_ch, frames) or NULL to generate it from F0
 * with the harmonic source (src/kokoro_modules.cpp:1574-1665). aff_in: NULL
 * (gamma, beta) = fc(style) for every AdaIN) or packed per-AdaIN blocks
 * [a][B][2*C_a] supplied by the caller (reference mode: the LoRA adapters sit
 * outside, src/decoder_lora.cpp:184-194). audio (B, hop*(frames-1)).
 * aff_out (optional) receives the resolved affines in the same packing.
 * Caches every intermediate the matching backward needs (inputs are copied);
 * params is borrowed: it must stay valid and unchanged until the matching
 * backward has been enqueued, as the reference's weights must outlive its
 * caches (include/brosoundml/decoder_lora.h:69-72). */
int bsml_decoder_forward(bsml_decoder* d, int B, int T, const float* params, const float* asr, const float* F0,
                         const float* N, const float* style, const float* har, int frames, const float* aff_in,
                         float* audio, float* aff_out, void* stream);

/* Inference: Kokoro::Impl::decode_back_half (src/kokoro.cpp:352-407), batched:
 * decoder backbone, harmonic source from F0, generator, iSTFT -> audio (B, S).
 * ref_s rows are ref_s_stride floats apart (2*style_dim for the reference's
 * (1, 2*style_dim) ref_s); the decoder reads the first style_dim of each row.
 * A backward may follow (it is the same forward). */
int bsml_decoder_decode(bsml_decoder* d, int B, int T, const float* params, const float* ref_s, int ref_s_stride,
                        const float* asr, const float* F0, const float* N, float* audio, void* stream);

/* Backward of the last forward. daudio (B, S). grads (n_params) is
 * OVERWRITTEN with d loss / d params (conv, convT, fc weights and biases,
 * Snake alphas). d_asr (B, asr_dim, T), d_style (B, style_dim), d_aff
 * (packed like aff_in) are optional outputs. In reference mode (aff_in given
 * to the forward) fc gradients and d_style are zero: the affines are inputs. */
int bsml_decoder_backward(bsml_decoder* d, const float* daudio, float* grads, float* d_asr, float* d_style,
                          float* d_aff, void* stream);

/* The two assemblies on their own, on a whole-decoder handle, batched over B
 * clips. The reference runs them as separate calls with caller-owned caches:
 * decoder_backbone_forward_train / _backward (src/kokoro_decoder_backward.h:213-231)
 * and generator_forward_train / generator_backward (:273-293). Here the engine
 * keeps the caches of its last forward.
 *   backbone:  asr (B, asr_dim, T), F0, N (B, 2T) -> gen_in (B, init_ch, L_gen),
 *              L_gen from bsml_backbone_out_len. The backward takes dgen_in and
 *              gives grads (n_params, OVERWRITTEN), d_asr, d_style, d_aff (optional).
 *   generator: gen_in (B, init_ch, L_in), har (B, har_ch, frames) -> audio
 *              (B, hop*(frames-1)). The backward takes daudio and gives grads,
 *              dgen_in (B, init_ch, L_in), d_style, d_aff (optional).
 * style rows are style_stride floats apart (0 = style_dim). aff_in / d_aff use
 * the whole decoder's packing; each part reads its own AdaINs and writes the
 * gradients of its own (the others' are zero). A backward follows the forward of
 * the same part. */
int bsml_backbone_out_len(const bsml_decoder* d, int T, int* L_gen);
int bsml_backbone_forward(bsml_decoder* d, int B, int T, const float* params, const float* asr, const float* F0,
                          const float* N, const float* style, int style_stride, const float* aff_in, float* gen_in,
                          float* aff_out, void* stream);
int bsml_backbone_backward(bsml_decoder* d, const float* dgen_in, float* grads, float* d_asr, float* d_style,
                           float* d_aff, void* stream);
int bsml_generator_forward(bsml_decoder* d, int B, int L_in, const float* params, const float* gen_in,
                           const float* har, int frames, const float* style, int style_stride, const float* aff_in,
                           float* audio, float* aff_out, void* stream);
int bsml_generator_backward(bsml_decoder* d, const float* daudio, float* grads, float* dgen_in, float* d_style,
                            float* d_aff, void* stream);

/* Bytes of device workspace the engine holds for the current (B, T). */
int64_t bsml_decoder_workspace_bytes(const bsml_decoder* d);

/* Optional per-kernel-class timing with CUDA events (no reference counterpart:
 * instrumentation for the roofline report). Classes (BSML_PROF_*): forward-like
 * convs (fwd, dgrad, convT) on the tensor cores and on the CUDA cores, weight
 * gradients on each, AdaIN+Snake forward, AdaIN+Snake backward. read_profile
 * fills 3 doubles per class (ms, algorithmic work in FLOPs for the convs or
 * bytes for the norms, launches), synchronises the device and clears the
 * record. */
enum {
    BSML_PROF_CONV_TC = 0, BSML_PROF_CONV_SIMT = 1, BSML_PROF_WGRAD_TC = 2, BSML_PROF_WGRAD_SIMT = 3,
    BSML_PROF_NORM_FWD = 4, BSML_PROF_NORM_BWD = 5, BSML_PROF_CLASSES = 6
};
int bsml_decoder_set_profiling(bsml_decoder* d, int on);
/* Number of CUDA kernels this library has launched in the process so far. */
int64_t bsml_launch_count(void);
/* out: 3 * BSML_PROF_CLASSES doubles */
int bsml_decoder_read_profile(bsml_decoder* d, double* out);
/* The same record launch by launch, in issue order: 3 doubles per launch (class,
 * work, ms), at most max_records; *n_records = how many were written. Clears the
 * record like read_profile. */
int bsml_decoder_read_profile_records(bsml_decoder* d, double* out, int max_records, int* n_records);

/* ── one decoder block on its own ──────────────────────────────────────────
 * The reference's block-level atoms, batched:
 *   BSML_BLOCK_RESBLK1D   detail::adain_resblk_1d_forward_train / _backward
 *                         (src/kokoro_decoder_backward.h:82-111): AdainResBlk1d
 *                         cin -> cout, optional x2 upsample (depthwise convT pool,
 *                         nearest-2x shortcut), learned 1x1 shortcut when cin != cout
 *   BSML_BLOCK_RESBLOCK1  detail::adain_resblock1_forward_train / _backward
 *                         (:125-144): AdaINResBlock1 with Snake, C channels, kernel,
 *                         convs1 dilations dil[3]
 * The handle is a bsml_decoder: param_count / param_table, set_math, profiling
 * and destroy apply; parameter keys are block-relative ("norm1.fc.weight",
 * "convs1.0.weight", "alpha2.1", ...). The whole-decoder entry points reject a
 * block handle and the block entry points reject a decoder handle. */
enum { BSML_BLOCK_RESBLK1D = 1, BSML_BLOCK_RESBLOCK1 = 2 };
typedef struct bsml_block_spec {
    int kind;        /* BSML_BLOCK_* */
    int style_dim;
    int cin, cout;   /* RESBLOCK1: cin = cout = C */
    int upsample;    /* RESBLK1D: 1 = x2 upsampling block */
    int kernel;      /* RESBLOCK1: odd conv kernel */
    int dil[3];      /* RESBLOCK1: convs1 dilations */
} bsml_block_spec;
int bsml_block_create(const bsml_block_spec* spec, int device, bsml_decoder** out);
/* Layout queries from a spec alone (no device needed). */
int bsml_block_param_count(const bsml_block_spec* spec, int64_t* n_params, int* n_entries, int* n_affine,
                           int64_t* aff_per_clip);
int bsml_block_param_table(const bsml_block_spec* spec, bsml_param_entry* out, int max_entries, int* aff_channels);
/* Forward: x (B, cin, L) NCL -> y (B, cout, L_out), L_out = 2L for an upsampling
 * AdainResBlk1d, else L. style (B, style_dim) or aff_in (packed [a][B][2*C_a],
 * adapter order: norm1, norm2 / adain1[0..2], adain2[0..2]). Caches what the
 * backward needs; params is borrowed until the backward has been enqueued. */
int bsml_block_forward(bsml_decoder* d, int B, int L, const float* params, const float* x, const float* style,
                       const float* aff_in, float* y, float* aff_out, void* stream);
/* Backward of the last block forward: dy (B, cout, L_out). grads (n_params)
 * OVERWRITTEN (optional); dx (B, cin, L), d_style, d_aff optional. */
int bsml_block_backward(bsml_decoder* d, const float* dy, float* grads, float* dx, float* d_style, float* d_aff,
                        void* stream);

/* ── safetensors (host-side IO; the reference's checkpoint format,
 * src/kokoro_modules.cpp:99-125) ─────────────────────────────────────────── */
typedef struct bsml_st bsml_st;
enum { BSML_ST_OTHER = 0, BSML_ST_F32 = 1, BSML_ST_F16 = 2, BSML_ST_BF16 = 3, BSML_ST_F64 = 4 };
int bsml_st_open(const char* path, bsml_st** out);
void bsml_st_close(bsml_st* f);
int bsml_st_count(const bsml_st* f, int* n);
/* i-th tensor in header order: name (NUL-terminated, truncated to name_cap),
 * dtype (BSML_ST_*), ndim and up to 8 dimensions. */
int bsml_st_info(const bsml_st* f, int i, char* name, int name_cap, int* dtype, int* ndim, int64_t* shape);
/* Reads tensor `name` into host memory as fp32 (F32, F16, BF16 or F64 sources);
 * n must equal its element count. */
int bsml_st_read_f32(const bsml_st* f, const char* name, float* dst, int64_t n);
/* __metadata__ string value of `key` (NUL-terminated, truncated to cap); error if absent. */
int bsml_st_metadata(const bsml_st* f, const char* key, char* value, int cap);
/* Fills the host parameter vector laid out by `table` (bsml_*_param_table) with
 * the tensors named prefix + entry name ("decoder.module." for a Kokoro
 * checkpoint). A weight held as weight_g / weight_v (PyTorch weight norm, the
 * unconverted upstream layout) is fused to g * v / ||v|| over all axes but the
 * first, as the reference's converter does (scripts/convert-kokoro.py:71-110).
 * Missing keys and size mismatches are errors. */
int bsml_params_from_safetensors(const bsml_st* f, const bsml_param_entry* table, int n_entries, const char* prefix,
                                 float* params, int64_t n_params);

/* ── data-parallel gradient averaging without torch ──────────────────────
 * One process per GPU. Rank 0 makes a 128-byte NCCL unique id and hands it to
 * the other ranks by any channel (a file, a socket, MPI); every rank then makes
 * its communicator and, each step, all-reduces its flat gradient buffer once
 * before the optimiser step. NCCL (2.14 or later) is loaded at run time
 * (libnccl.so.2). No reference counterpart: the reference has no multi-GPU path.
 *
 * Failure handling: the communicator is non-blocking and carries a timeout.
 * Set-up returns an error when the other ranks do not join within it;
 * bsml_nccl_sync waits for a step's collectives and, when they do not finish
 * within it (a peer left between steps) or NCCL reports an error, aborts the
 * communicator (ending its kernels still waiting on the GPU) and returns an
 * error. An aborted communicator rejects further use; destroy it. */
#define BSML_NCCL_DEFAULT_TIMEOUT_MS 120000
int bsml_nccl_unique_id(void* id /* 128 bytes */);
int bsml_nccl_version(int* version);
int bsml_nccl_comm_init(int nranks, const void* id, int rank, int device, void** comm);
int bsml_nccl_comm_init_timeout(int nranks, const void* id, int rank, int device, int timeout_ms, void** comm);
int bsml_nccl_comm_destroy(void* comm);
/* grads (n floats, device) summed over the ranks, or averaged when average != 0.
 * Asynchronous on stream. */
int bsml_allreduce_grads(void* comm, float* grads, int64_t n, int average, void* stream);
/* Blocks the host until stream is idle, bounded by the communicator's timeout. */
int bsml_nccl_sync(void* comm, void* stream);

/* ── CUDA graphs (no reference counterpart: the reference runs eagerly) ────
 * Records every library call issued on `stream` between begin and end (a whole
 * forward, loss and backward, say) into one CUDA graph; launch replays it with
 * the same pointers and shapes, so new data is written into the same input
 * buffers between launches. Run the same sequence once eagerly first: the first
 * call of a shape plans and allocates the engine's workspace, which a capture
 * cannot do. stream must not be the legacy default stream. Keep an optimiser
 * step with a step count outside the graph (its count is a launch argument). */
typedef struct bsml_graph bsml_graph;
int bsml_graph_begin(void* stream);
int bsml_graph_end(void* stream, bsml_graph** out);
int bsml_graph_launch(bsml_graph* g, void* stream);
/* Kernel nodes in the graph (the launches one replay issues). */
int bsml_graph_kernel_count(const bsml_graph* g, int64_t* n);
void bsml_graph_destroy(bsml_graph* g);

/* ── loss and optimiser ─────────────────────────────────────────────────── */

/* L1 loss: loss[0] = mean |audio - target|, daudio = sign(audio - target) / n. */
int bsml_loss_l1(const float* audio, const float* target, int64_t n, float* loss, float* daudio, void* stream);

/* Adam with bias correction, in place over n floats (bt::adam_step as used by
 * DecoderLora::adam_step, src/decoder_lora.cpp:306-314). */
int bsml_adam_step(float* param, const float* grad, float* m, float* v, int64_t n, float lr, float beta1,
                   float beta2, float eps, int step, void* stream);

/* ── DecoderLora (include/brosoundml/decoder_lora.h:36-164) ─────────────────
 * LoRA adapters on every AdaIN's style -> (gamma, beta) fc, a shared
 * conditioning gate g(v) = W2 tanh(W1 v) (in_dim 3, hidden 16, width = rank,
 * W2 zero at creation), Adam and the ELRA1 checkpoint; batched over clips (the
 * reference runs one clip). The decoder runs in reference mode under it: the
 * base weights are frozen and no weight gradients are formed. A bsml_lora
 * refers to its bsml_decoder and must be destroyed first. */
typedef struct bsml_lora bsml_lora;

/* DecoderLora::make (src/decoder_lora.cpp:115-147): rank 1..32, LoRA scale,
 * seed (0 = the reference default) for the xavier-uniform A, B and gate W1. */
int bsml_lora_create(bsml_decoder* d, int rank, float scale, uint64_t seed, bsml_lora** out);
void bsml_lora_destroy(bsml_lora* l);
/* Sizes. The flat parameter vector (device; gradients share the layout) holds
 * gate W1 [16][3], gate W2 [rank][16], then per adapter (adapters() order)
 * A [rank][style_dim] and B [2C][rank]. off_A / off_B: n_adapters entries each. */
int bsml_lora_layout(const bsml_lora* l, int64_t* n_params, int* n_adapters, int* rank, int* style_dim,
                     int64_t* off_W1, int64_t* off_W2, int64_t* off_A, int64_t* off_B, int* adapter_C);
/* Device pointers to the parameter and gradient vectors (owned by the object). */
int bsml_lora_buffers(bsml_lora* l, float** params, float** grads);
/* Adam's first and second moments (device; the parameter vector's layout). */
int bsml_lora_moments(bsml_lora* l, float** m, float** v);
/* ConditioningGate on its own (src/decoder_lora.cpp:28-78), batched over B
 * condition vectors v (B, in_dim): act = tanh(W1 v) (B, hidden), g = W2 act
 * (B, gate_dim); W1 (hidden, in_dim), W2 (gate_dim, hidden), no biases. The
 * backward ACCUMULATES dW1, dW2 (+=) from dG (B, gate_dim), like the reference's
 * gradient accumulators (zero them between steps). hidden, gate_dim <= 64. */
int bsml_gate_forward(const float* W1, const float* W2, const float* v, int B, int in_dim, int hidden, int gate_dim,
                      float* act, float* g, void* stream);
int bsml_gate_backward(const float* W2, const float* v, const float* act, const float* dG, int B, int in_dim,
                       int hidden, int gate_dim, float* dW1, float* dW2, void* stream);
/* DecoderLora::forward (src/decoder_lora.cpp:211-246), batched: style of clip b
 * = ref_s[b*ref_s_stride .. + style_dim), cond (B, 3), har optional (NULL: the
 * harmonic source). params = the frozen decoder weights, borrowed until the
 * matching backward. */
int bsml_lora_forward(bsml_lora* l, int B, int T, const float* params, const float* asr, const float* F0,
                      const float* N, const float* ref_s, int ref_s_stride, const float* har, int frames,
                      const float* cond, float* audio, void* stream);
/* DecoderLora::backward (src/decoder_lora.cpp:248-296): accumulates the adapter
 * and gate gradients (until bsml_lora_zero_grad). */
int bsml_lora_backward(bsml_lora* l, const float* daudio, void* stream);
int bsml_lora_zero_grad(bsml_lora* l, void* stream);
/* DecoderLora::adam_step: one shared step count for every tensor. */
int bsml_lora_adam_step(bsml_lora* l, float lr, float beta1, float beta2, float eps, void* stream);
/* DecoderLora::save / load (src/decoder_lora.cpp:324-396): the ELRA1 byte
 * format; load restores values into an object of the same architecture and
 * takes the scale from the file. Synchronous. */
int bsml_lora_save(const bsml_lora* l, const char* path);
int bsml_lora_load(bsml_lora* l, const char* path);
/* Full training state (no reference counterpart; the reference drops the
 * optimiser state): the ELRA1 file followed by Adam's moments and step, so a
 * reader of the plain format (bsml_lora_load or the reference's
 * DecoderLora::load, which stops after the last adapter) still reads it;
 * load_state restores parameters, moments and step. Synchronous. */
int bsml_lora_save_state(const bsml_lora* l, const char* path);
int bsml_lora_load_state(bsml_lora* l, const char* path);
/* Current LoRA scale and Adam step count. */
int bsml_lora_state(const bsml_lora* l, float* scale, int* step);

/* ── conv-weight LoRA (no counterpart in the reference) ─────────────────────
 * A rank-r adapter on every Conv1d / ConvTranspose1d weight, base weights frozen.
 * A weight stored (d0, d1, k) is viewed as [d0][d1*k] and adapted to
 * W + scale * B A, A [rank][d1*k] ~ N(0, 0.01) at creation, B [d0][rank] = 0.
 * Refers to its bsml_decoder, which must outlive it. */
typedef struct bsml_convlora bsml_convlora;

int bsml_convlora_create(bsml_decoder* d, int rank, float scale, uint64_t seed, bsml_convlora** out);
void bsml_convlora_destroy(bsml_convlora* l);
/* n_weights adapted weights; per weight (arrays of n_weights): its offset in the
 * decoder parameters, rows (d0), cols (d1*k), and the offsets of A and B in the
 * flat LoRA parameter vector. */
int bsml_convlora_layout(const bsml_convlora* l, int64_t* n_params, int* n_weights, int64_t* w_off, int* rows,
                         int* cols, int64_t* off_A, int64_t* off_B);
int bsml_convlora_buffers(bsml_convlora* l, float** params, float** grads);
/* Forward of the adapted decoder; params = the frozen base weights (read during
 * the call only: the adapters are folded into a private copy). */
int bsml_convlora_forward(bsml_convlora* l, int B, int T, const float* params, const float* asr, const float* F0,
                          const float* N, const float* style, const float* har, int frames, float* audio,
                          void* stream);
/* Accumulates dA, dB from the audio gradient (until bsml_convlora_zero_grad). */
int bsml_convlora_backward(bsml_convlora* l, const float* daudio, void* stream);
int bsml_convlora_zero_grad(bsml_convlora* l, void* stream);
int bsml_convlora_adam_step(bsml_convlora* l, float lr, float beta1, float beta2, float eps, void* stream);
/* Full training state in the ECLR1 format: magic "ECLR1\0\0\0", int32 rank,
 * float scale, int32 n_weights, per weight (int64 offset, int32 rows, int32 cols),
 * int32 Adam step, int64 n_params, then parameters, first and second moments
 * (float32 each). load checks the architecture. Synchronous. */
int bsml_convlora_save(const bsml_convlora* l, const char* path);
int bsml_convlora_load(bsml_convlora* l, const char* path);

/* ── atoms (the reference's detail:: functions, batched) ────────────────── */

/* Arithmetic of the conv / convT atoms below (process-wide, default
 * BSML_MATH_FP32_SIMT). Tensor-core modes apply to stride-1 contractions with
 * >= 32 input and >= 64 output channels; others stay on the fp32 kernels. */
int bsml_set_atom_math(int math_mode);
/* Reads and clears the error word a tensor-core kernel sets when one of its
 * bounded waits gives up (0 = none). Synchronises the device. */
int bsml_device_error(void);
/* Debug builds (make -C brosoundml_b200 DEBUG=1, a separate libbsml_b200_debug.so;
 * no reference counterpart) check every channels-last row access of the
 * elementwise, normalisation and spectral kernels: the first access outside its
 * view is recorded and clamped into range. record[0..4] = (1, b, l, B, L) of that
 * access, or zeros (always zeros in release builds); reading clears it and
 * synchronises the device. */
int bsml_debug_bounds(int* record);
/* Self-test of that mechanism (no reference counterpart): launches one kernel
 * whose bounded wait, on a barrier nothing completes, gives up after about 2 s
 * and leaves code 1 (wait for data) in the error word; the context stays usable. */
int bsml_selftest_bounded_wait(void* stream);

/* Conv1d forward (modules.cpp:103-108): x (B, Ci, L) -> y (B, Co, Lo). bias may be NULL. */
int bsml_conv1d_forward(const float* x, int B, int Ci, int L, const float* W, const float* bias, int Co, int k,
                        int stride, int pad, int dil, float* y, void* stream);
/* conv1d_backward_input (kokoro_decoder_backward.cpp:230-234): dy (B, Co, Lo) -> dx (B, Ci, L). stride 1. */
int bsml_conv1d_backward_input(const float* dy, int B, int Ci, int L, const float* W, int Co, int k, int stride,
                               int pad, int dil, float* dx, void* stream);
/* Weight / bias gradient (overwritten). db may be NULL. */
int bsml_conv1d_backward_weight(const float* dy, const float* x, int B, int Ci, int L, int Co, int k, int stride,
                                int pad, int dil, float* dW, float* db, void* stream);
/* Conv1d weight / bias gradient that allocates nothing. No counterpart in the
 * reference: it is for callers that may not call cudaMalloc while computing
 * gradients (a real-time audio thread that must not block on the driver's
 * allocator, or an application whose device memory is all reserved up front by
 * its own arena). Same arguments and results as bsml_conv1d_backward_weight, but
 * its scratch (channels-last copies of dy and x, split-K partial sums) lives in
 * one static device array of BSML_NOALLOC_SCRATCH_FLOATS floats (16 MiB) that
 * every GPU loading this library holds until exit. A problem whose scratch
 * (B*Lo*round_up(Co,4) + B*L*round_up(Ci,4) + Co*Ci*k floats, roughly) exceeds
 * it is rejected with an error. The first call on each device looks the array's
 * device address up (cudaGetSymbolAddress): make that first call before any
 * stream capture. All calls share the array, so calls that overlap on the GPU
 * (other streams, other threads) race; serialise them on one stream. */
#define BSML_NOALLOC_SCRATCH_FLOATS (4ll * 1024 * 1024)
int bsml_conv1d_backward_weight_noalloc(const float* dy, const float* x, int B, int Ci, int L, int Co, int k,
                                        int stride, int pad, int dil, float* dW, float* db, void* stream);

/* ConvTranspose1d, groups 1, output_padding 0 (kokoro_decoder_backward.cpp:627-629): W (Ci, Co, k). */
int bsml_conv_transpose1d_forward(const float* x, int B, int Ci, int L, const float* W, const float* bias, int Co,
                                  int k, int stride, int pad, float* y, void* stream);
int bsml_conv_transpose1d_backward_input(const float* dy, int B, int Ci, int L, const float* W, int Co, int k,
                                         int stride, int pad, float* dx, void* stream);
int bsml_conv_transpose1d_backward_weight(const float* dy, const float* x, int B, int Ci, int L, int Co, int k,
                                          int stride, int pad, float* dW, float* db, void* stream);

/* adain_affine_forward / _backward (kokoro_decoder_backward.h:37-56), batched:
 * x (B, C, L), gb (B, 2C) = (gamma ; beta) per clip. dgb overwritten. */
int bsml_adain_affine_forward(const float* x, const float* gb, int B, int C, int L, float eps, float* y,
                              void* stream);
int bsml_adain_affine_backward(const float* x, const float* gb, const float* dy, int B, int C, int L, float eps,
                               float* dx, float* dgb, void* stream);
/* Snake1D (kokoro_modules.h:253) and its backward with the alpha gradient (overwritten). */
int bsml_snake_forward(const float* x, const float* alpha, int B, int C, int L, float* y, void* stream);
int bsml_snake_backward(const float* x, const float* alpha, const float* dy, int B, int C, int L, float* dx,
                        float* dalpha, void* stream);
/* iSTFT (center, periodic Hann n_fft, length hop*(L-1)) and its adjoint; re/im (B, n_fft/2+1, L). */
int bsml_istft_forward(const float* re, const float* im, int B, int n_fft, int hop, int L, float* audio,
                       void* stream);
int bsml_istft_backward(const float* daudio, int B, int n_fft, int hop, int L, float* dre, float* dim,
                        void* stream);
/* spectral_head_forward_train / _backward (src/kokoro_decoder_backward.h:145-161),
 * batched: x (B, C, L) -> leaky 0.01 -> conv_post (W (n_fft+2, C, post_kernel),
 * bias or NULL, padding (post_kernel-1)/2) -> post (B, n_fft+2, L), the cache the
 * backward reads -> mag = exp(post[:nf]), phase = sin(post[nf:]) -> iSTFT (center,
 * periodic Hann of n_fft, hop) -> audio (B, hop*(L-1)). The backward maps daudio
 * to dx (B, C, L) given the forward's x and post (conv_post frozen, as in the
 * reference). */
int bsml_spectral_head_forward(const float* x, int B, int C, int L, const float* W, const float* bias, int n_fft,
                               int hop, int post_kernel, float* post, float* audio, void* stream);
int bsml_spectral_head_backward(const float* x, const float* post, const float* daudio, int B, int C, int L,
                                const float* W, int n_fft, int hop, int post_kernel, float* dx, void* stream);
/* (batch, rows, cols) -> (batch, cols, rows): NCL <-> the reference's (L, C)
 * sequence layout (bt::nchw_to_sequence, kokoro_decoder_backward.cpp:112-116). */
int bsml_transpose(const float* src, int64_t batch, int rows, int cols, float* dst, void* stream);

/* Memory for callers that keep host-addressable tensors (the reference's
 * brotensor::Tensor is read and written element by element on the host, e.g. by
 * its finite-difference tests): CUDA managed memory, zero-filled. bsml_memcpy
 * copies between any two addresses the device can reach. */
int bsml_managed_alloc(int64_t bytes, void** out);
int bsml_managed_free(void* p);
int bsml_synchronize(void);
int bsml_memcpy(void* dst, const void* src, int64_t bytes, void* stream);

/* HarmonicSource::forward (kokoro_modules.cpp:1574-1665): F0 (B, F) -> har (B, n_fft+2, F*scale/hop+1).
 * Phase arithmetic: BSML_PHASE_FP32_RUNNING is the reference's own (one fp32
 * accumulator per harmonic, per-sample add and a single 2*pi subtraction,
 * kokoro_modules.cpp:1601-1616), reproduced bit for bit; the default.
 * BSML_PHASE_EXACT forms every frame's start phase exactly (double), a sine
 * source whose phase does not drift over long clips (not the reference's). */
enum { BSML_PHASE_FP32_RUNNING = 0, BSML_PHASE_EXACT = 1 };
int bsml_harmonic_source(const bsml_decoder_config* cfg, const float* F0, int B, int F, const float* l_weight,
                         const float* l_bias, float* har, void* stream);
int bsml_harmonic_source_mode(const bsml_decoder_config* cfg, const float* F0, int B, int F, const float* l_weight,
                              const float* l_bias, float* har, int phase_mode, void* stream);
/* The phase mode of the harmonic source a decoder runs when no har is passed. */
int bsml_decoder_set_phase_mode(bsml_decoder* d, int phase_mode);

#ifdef __cplusplus
}
#endif

#endif /* BSML_DECODER_H */
