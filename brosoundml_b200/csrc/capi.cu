// extern "C" boundary (include/bsml_decoder.h). Every entry point converts
// exceptions into a negative status and a thread-local message.
#include <cstring>
#include <memory>
#include <string>

#include <atomic>

#include "bsml_decoder.h"
#include "conv_tc.h"
#include "engine.h"
#include "kernels.h"
#include "convlora.h"
#include "lora.h"
#include "nccl_dl.h"
#include "safetensors.h"

namespace {

thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    } catch (...) {
        g_err = "brosoundml: unknown error";
        return -1;
    }
}

cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Stream-ordered scratch for the atom entry points (which, like the reference's
// detail:: atoms, own their temporaries).
struct Scratch {
    cudaStream_t st;
    std::vector<void*> ptrs;
    explicit Scratch(cudaStream_t s) : st(s) {}
    float* f(int64_t n) {
        void* p = nullptr;
        bsml::check_cuda(cudaMallocAsync(&p, std::max<int64_t>(n, 1) * 4, st), "cudaMallocAsync");
        ptrs.push_back(p);
        return (float*)p;
    }
    double* d(int64_t n) {
        void* p = nullptr;
        bsml::check_cuda(cudaMallocAsync(&p, std::max<int64_t>(n, 1) * 8, st), "cudaMallocAsync");
        ptrs.push_back(p);
        return (double*)p;
    }
    bsml::Act act(int B, int L, int C) {
        bsml::Act a;
        a.B = B; a.L = L; a.C = C; a.ld = bsml::pitch(C);
        a.bstride = (int64_t)L * a.ld;
        a.p = f((int64_t)B * a.bstride);
        return a;
    }
    ~Scratch() {
        for (void* p : ptrs) cudaFreeAsync(p, st);
    }
};

void need(bool ok, const char* where, const char* why) {
    if (!ok) bsml::fail(where, why);
}

// an inner C-ABI call's failure re-raised with its own message
void check_rc(int rc) {
    if (rc != 0) throw std::runtime_error(g_err);
}

// output length of a conv; 0 (rejected by the callers) when the padded input is
// shorter than the dilated kernel (a negative numerator must not truncate to 0)
int conv_out(int L, int k, int s, int p, int d) {
    const int64_t num = (int64_t)L + 2 * (int64_t)p - (int64_t)d * (k - 1) - 1;
    return (num < 0 || s <= 0) ? 0 : (int)(num / s + 1);
}

std::atomic<int> g_atom_math{BSML_MATH_FP32_SIMT};

bool atom_tc(int K, int M, int s) { return g_atom_math.load() != BSML_MATH_FP32_SIMT && s == 1 && K >= 32 && M >= 64; }
// ConvTranspose1d gradients on the tensor cores: dy viewed row-packed (K = s*Co per tap)
bool atom_convT_tc(int Ci, int Co, int s, int Lu) {
    return g_atom_math.load() != BSML_MATH_FP32_SIMT && Ci >= 64 && s * Co >= 32 && Co % 8 == 0 && Lu % s == 0;
}
int atom_tc_mode() {
    const int m = g_atom_math.load();
    return m == BSML_MATH_BF16 ? bsml::TC_BF16 : m == BSML_MATH_BF16X3 ? bsml::TC_BF16X3 : bsml::TC_TF32X3;
}
// input gradients: BF16X3 under TF32X3F; weight gradients: BF16X3 under TF32X3W and
// TF32X3F; else the mode above
int atom_dg_mode() { return g_atom_math.load() == BSML_MATH_TF32X3F ? bsml::TC_BF16X3 : atom_tc_mode(); }
int atom_wg_mode() {
    const int m = g_atom_math.load();
    return (m == BSML_MATH_TF32X3W || m == BSML_MATH_TF32X3F) ? bsml::TC_BF16X3 : atom_tc_mode();
}

// Tensor-core forward-like conv for the atoms: planes of x, packed weight planes, launch.
void atom_tc_conv(Scratch& sc, const bsml::Act& xa, const float* W, int kind, int Co_w, int Ci_w, int k, int s_ph,
                  int r_ph, int taps, int M, const bsml::Act& ya, const float* bias, int p, int d, int No, int o_base,
                  int orow_mul, int orow_off, cudaStream_t st, int mode = -1) {
    if (mode < 0) mode = atom_tc_mode();
    float* xh = sc.f((int64_t)xa.B * xa.L * bsml::tc_pitch(xa.C, mode));
    float* xl = sc.f((int64_t)xa.B * xa.L * bsml::tc_pitch(xa.C, mode));
    const int64_t wn = (int64_t)taps * M * bsml::round_up(xa.C, 8);
    float* wh = sc.f(wn);
    float* wl = sc.f(wn);
    bsml::make_act_planes(xa, mode, xh, xl, st);
    bsml::pack_w_tc(W, kind, Co_w, Ci_w, k, s_ph, r_ph, mode, wh, wl, st);
    bsml::TcConvFwd a;
    a.x.hi = xh; a.x.lo = xl; a.x.ld = bsml::tc_pitch(xa.C, mode);
    a.B = xa.B; a.L_in = xa.L; a.Ci = xa.C;
    a.w.hi = wh; a.w.lo = wl; a.w.ld = (int)bsml::round_up(xa.C, 8);
    a.taps = taps; a.Co = M; a.p = p; a.d = d; a.No = No; a.o_base = o_base;
    a.y = ya; a.bias = bias; a.orow_mul = orow_mul; a.orow_off = orow_off;
    a.part_cap = bsml::conv_fwd_tc_part_floats(a, mode);
    if (a.part_cap > 0) a.part = sc.f(a.part_cap);
    bsml::conv_fwd_tc(a, mode, st);
}

}  // namespace

void bsml::set_last_error(const std::string& msg) { g_err = msg; }

struct bsml_decoder {
    std::unique_ptr<bsml::Engine> eng;
};

struct bsml_lora {
    std::unique_ptr<bsml::Lora> lora;
};

struct bsml_convlora {
    std::unique_ptr<bsml::ConvLora> lora;
};

extern "C" {

const char* bsml_last_error(void) { return g_err.c_str(); }
int bsml_version(void) { return 1; }

int bsml_decoder_create(const bsml_decoder_config* cfg, int device, bsml_decoder** out) {
    return guarded([&] {
        need(cfg && out, "bsml_decoder_create", "null argument");
        auto* d = new bsml_decoder;
        try {
            d->eng = std::make_unique<bsml::Engine>(*cfg, device);
        } catch (...) {
            delete d;
            throw;
        }
        *out = d;
    });
}

void bsml_decoder_destroy(bsml_decoder* d) { delete d; }

int bsml_decoder_param_count(const bsml_decoder* d, int64_t* n_params, int* n_entries, int* n_affine,
                             int64_t* aff_per_clip) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_param_count", "null handle");
        const auto& L = d->eng->layout();
        if (n_params) *n_params = L.total;
        if (n_entries) *n_entries = (int)L.table.size();
        if (n_affine) *n_affine = (int)L.aff_C.size();
        if (aff_per_clip) *aff_per_clip = L.aff_per_clip;
    });
}

int bsml_decoder_param_table(const bsml_decoder* d, bsml_param_entry* out, int max_entries, int* aff_channels) {
    int n = 0;
    const int rc = guarded([&] {
        need(d != nullptr, "bsml_decoder_param_table", "null handle");
        const auto& L = d->eng->layout();
        n = std::min<int>(max_entries, (int)L.table.size());
        for (int i = 0; i < n; ++i) out[i] = L.table[i];
        if (aff_channels)
            for (size_t i = 0; i < L.aff_C.size(); ++i) aff_channels[i] = L.aff_C[i];
    });
    return rc ? rc : n;
}

int bsml_config_param_count(const bsml_decoder_config* cfg, int64_t* n_params, int* n_entries, int* n_affine,
                            int64_t* aff_per_clip) {
    return guarded([&] {
        need(cfg != nullptr, "bsml_config_param_count", "null config");
        const bsml::Layout L(*cfg);
        if (n_params) *n_params = L.total;
        if (n_entries) *n_entries = (int)L.table.size();
        if (n_affine) *n_affine = (int)L.aff_C.size();
        if (aff_per_clip) *aff_per_clip = L.aff_per_clip;
    });
}

int bsml_config_param_table(const bsml_decoder_config* cfg, bsml_param_entry* out, int max_entries,
                            int* aff_channels) {
    int n = 0;
    const int rc = guarded([&] {
        need(cfg != nullptr && out != nullptr, "bsml_config_param_table", "null argument");
        const bsml::Layout L(*cfg);
        n = std::min<int>(max_entries, (int)L.table.size());
        for (int i = 0; i < n; ++i) out[i] = L.table[i];
        if (aff_channels)
            for (size_t i = 0; i < L.aff_C.size(); ++i) aff_channels[i] = L.aff_C[i];
    });
    return rc ? rc : n;
}

int bsml_decoder_set_math(bsml_decoder* d, int math_mode) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_set_math", "null handle");
        d->eng->set_math(math_mode);
    });
}

int bsml_decoder_forward(bsml_decoder* d, int B, int T, const float* params, const float* asr, const float* F0,
                         const float* N, const float* style, const float* har, int frames, const float* aff_in,
                         float* audio, float* aff_out, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_forward", "null handle");
        d->eng->forward(B, T, params, asr, F0, N, style, har, frames, aff_in, audio, aff_out, S(stream));
    });
}

int bsml_decoder_decode(bsml_decoder* d, int B, int T, const float* params, const float* ref_s, int ref_s_stride,
                        const float* asr, const float* F0, const float* N, float* audio, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_decode", "null handle");
        need(ref_s != nullptr, "bsml_decoder_decode", "null ref_s");
        d->eng->forward(B, T, params, asr, F0, N, ref_s, nullptr, 0, nullptr, audio, nullptr, S(stream),
                        ref_s_stride);
    });
}

int bsml_decoder_backward(bsml_decoder* d, const float* daudio, float* grads, float* d_asr, float* d_style,
                          float* d_aff, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_backward", "null handle");
        d->eng->backward(daudio, grads, d_asr, d_style, d_aff, S(stream));
    });
}

int bsml_backbone_out_len(const bsml_decoder* d, int T, int* L_gen) {
    return guarded([&] {
        need(d != nullptr && L_gen != nullptr && T > 0, "bsml_backbone_out_len", "bad argument");
        *L_gen = d->eng->backbone_out_len(T);
    });
}

int bsml_backbone_forward(bsml_decoder* d, int B, int T, const float* params, const float* asr, const float* F0,
                          const float* N, const float* style, int style_stride, const float* aff_in, float* gen_in,
                          float* aff_out, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_backbone_forward", "null handle");
        d->eng->forward_backbone(B, T, params, asr, F0, N, style, style_stride, aff_in, gen_in, aff_out, S(stream));
    });
}

int bsml_backbone_backward(bsml_decoder* d, const float* dgen_in, float* grads, float* d_asr, float* d_style,
                           float* d_aff, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_backbone_backward", "null handle");
        d->eng->backward_backbone(dgen_in, grads, d_asr, d_style, d_aff, S(stream));
    });
}

int bsml_generator_forward(bsml_decoder* d, int B, int L_in, const float* params, const float* gen_in,
                           const float* har, int frames, const float* style, int style_stride, const float* aff_in,
                           float* audio, float* aff_out, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_generator_forward", "null handle");
        d->eng->forward_generator(B, L_in, params, gen_in, har, frames, style, style_stride, aff_in, audio, aff_out,
                                  S(stream));
    });
}

int bsml_generator_backward(bsml_decoder* d, const float* daudio, float* grads, float* dgen_in, float* d_style,
                            float* d_aff, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_generator_backward", "null handle");
        d->eng->backward_generator(daudio, grads, dgen_in, d_style, d_aff, S(stream));
    });
}

int bsml_block_create(const bsml_block_spec* spec, int device, bsml_decoder** out) {
    return guarded([&] {
        need(spec && out, "bsml_block_create", "null argument");
        auto* d = new bsml_decoder;
        try {
            d->eng = std::make_unique<bsml::Engine>(*spec, device);
        } catch (...) {
            delete d;
            throw;
        }
        *out = d;
    });
}

int bsml_block_param_count(const bsml_block_spec* spec, int64_t* n_params, int* n_entries, int* n_affine,
                           int64_t* aff_per_clip) {
    return guarded([&] {
        need(spec != nullptr, "bsml_block_param_count", "null spec");
        const bsml::Layout L(*spec);
        if (n_params) *n_params = L.total;
        if (n_entries) *n_entries = (int)L.table.size();
        if (n_affine) *n_affine = (int)L.aff_C.size();
        if (aff_per_clip) *aff_per_clip = L.aff_per_clip;
    });
}

int bsml_block_param_table(const bsml_block_spec* spec, bsml_param_entry* out, int max_entries, int* aff_channels) {
    int n = 0;
    const int rc = guarded([&] {
        need(spec != nullptr && out != nullptr, "bsml_block_param_table", "null argument");
        const bsml::Layout L(*spec);
        n = std::min<int>(max_entries, (int)L.table.size());
        for (int i = 0; i < n; ++i) out[i] = L.table[i];
        if (aff_channels)
            for (size_t i = 0; i < L.aff_C.size(); ++i) aff_channels[i] = L.aff_C[i];
    });
    return rc ? rc : n;
}

int bsml_block_forward(bsml_decoder* d, int B, int L, const float* params, const float* x, const float* style,
                       const float* aff_in, float* y, float* aff_out, void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_block_forward", "null handle");
        d->eng->forward_block(B, L, params, x, style, aff_in, y, aff_out, S(stream));
    });
}

int bsml_block_backward(bsml_decoder* d, const float* dy, float* grads, float* dx, float* d_style, float* d_aff,
                        void* stream) {
    return guarded([&] {
        need(d != nullptr, "bsml_block_backward", "null handle");
        d->eng->backward_block(dy, grads, dx, d_style, d_aff, S(stream));
    });
}

int64_t bsml_decoder_workspace_bytes(const bsml_decoder* d) { return d ? d->eng->workspace_bytes() : 0; }

int64_t bsml_launch_count(void) { return bsml::launch_count(); }

int bsml_set_atom_math(int math_mode) {
    return guarded([&] {
        need(math_mode == BSML_MATH_FP32_SIMT || math_mode == BSML_MATH_TF32X3 || math_mode == BSML_MATH_BF16 ||
                 math_mode == BSML_MATH_BF16X3 || math_mode == BSML_MATH_TF32X3W || math_mode == BSML_MATH_TF32X3F,
             "bsml_set_atom_math", "unknown math mode");
        g_atom_math.store(math_mode);
    });
}

#ifdef BSML_DEBUG_BOUNDS
}  // extern "C"
namespace bsml {
__device__ int g_dbg_bounds[5];
}
extern "C" {
#endif

int bsml_debug_bounds(int* record) {
    return guarded([&] {
        need(record != nullptr, "bsml_debug_bounds", "null argument");
        for (int i = 0; i < 5; ++i) record[i] = 0;
#ifdef BSML_DEBUG_BOUNDS
        BSML_CUDA(cudaDeviceSynchronize());
        BSML_CUDA(cudaMemcpyFromSymbol(record, bsml::g_dbg_bounds, sizeof(int) * 5));
        const int zero[5] = {0, 0, 0, 0, 0};
        BSML_CUDA(cudaMemcpyToSymbol(bsml::g_dbg_bounds, zero, sizeof(zero)));
#endif
    });
}

int bsml_device_error(void) {
    int v = 0;
    const int rc = guarded([&] { v = bsml::tc_error_flag(); });
    return rc ? rc : v;
}

int bsml_selftest_bounded_wait(void* stream) {
    return guarded([&] { bsml::tc_wait_selftest(S(stream)); });
}

int bsml_decoder_set_profiling(bsml_decoder* d, int on) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_set_profiling", "null handle");
        d->eng->set_profiling(on != 0);
    });
}

int bsml_decoder_read_profile(bsml_decoder* d, double* out) {
    return guarded([&] {
        need(d != nullptr && out != nullptr, "bsml_decoder_read_profile", "null argument");
        d->eng->read_profile(out);
    });
}

int bsml_decoder_read_profile_records(bsml_decoder* d, double* out, int max_records, int* n_records) {
    return guarded([&] {
        need(d != nullptr && out != nullptr && n_records != nullptr && max_records >= 0,
             "bsml_decoder_read_profile_records", "bad argument");
        d->eng->read_profile_records(out, max_records, n_records);
    });
}

int bsml_lora_create(bsml_decoder* d, int rank, float scale, uint64_t seed, bsml_lora** out) {
    return guarded([&] {
        need(d && out, "bsml_lora_create", "null argument");
        auto* l = new bsml_lora;
        try {
            l->lora = std::make_unique<bsml::Lora>(*d->eng, rank, scale, seed);
        } catch (...) {
            delete l;
            throw;
        }
        *out = l;
    });
}

void bsml_lora_destroy(bsml_lora* l) { delete l; }

int bsml_lora_layout(const bsml_lora* l, int64_t* n_params, int* n_adapters, int* rank, int* style_dim,
                     int64_t* off_W1, int64_t* off_W2, int64_t* off_A, int64_t* off_B, int* adapter_C) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_layout", "null handle");
        const bsml::Lora& L = *l->lora;
        if (n_params) *n_params = L.n_params();
        if (n_adapters) *n_adapters = L.n_adapters();
        if (rank) *rank = L.rank();
        if (style_dim) *style_dim = L.style_dim();
        if (off_W1) *off_W1 = L.off_W1();
        if (off_W2) *off_W2 = L.off_W2();
        for (int a = 0; a < L.n_adapters(); ++a) {
            if (off_A) off_A[a] = L.adapters()[a].offA;
            if (off_B) off_B[a] = L.adapters()[a].offB;
            if (adapter_C) adapter_C[a] = L.adapters()[a].C;
        }
    });
}

int bsml_lora_buffers(bsml_lora* l, float** params, float** grads) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_buffers", "null handle");
        if (params) *params = l->lora->params();
        if (grads) *grads = l->lora->grads();
    });
}

int bsml_lora_moments(bsml_lora* l, float** m, float** v) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_moments", "null handle");
        if (m) *m = l->lora->moment1();
        if (v) *v = l->lora->moment2();
    });
}

int bsml_gate_forward(const float* W1, const float* W2, const float* v, int B, int in_dim, int hidden, int gate_dim,
                      float* act, float* g, void* stream) {
    return guarded([&] {
        need(W1 && W2 && v && act && g && B > 0 && in_dim > 0 && hidden > 0 && gate_dim > 0, "bsml_gate_forward",
             "bad argument");
        bsml::gate_forward(W1, W2, v, B, in_dim, hidden, gate_dim, act, g, S(stream));
    });
}

int bsml_gate_backward(const float* W2, const float* v, const float* act, const float* dG, int B, int in_dim,
                       int hidden, int gate_dim, float* dW1, float* dW2, void* stream) {
    return guarded([&] {
        need(W2 && v && act && dG && dW1 && dW2 && B > 0 && in_dim > 0 && hidden > 0 && gate_dim > 0,
             "bsml_gate_backward", "bad argument");
        bsml::gate_backward(W2, v, act, dG, B, in_dim, hidden, gate_dim, dW1, dW2, S(stream));
    });
}

int bsml_lora_forward(bsml_lora* l, int B, int T, const float* params, const float* asr, const float* F0,
                      const float* N, const float* ref_s, int ref_s_stride, const float* har, int frames,
                      const float* cond, float* audio, void* stream) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_forward", "null handle");
        l->lora->forward(B, T, params, asr, F0, N, ref_s, ref_s_stride, har, frames, cond, audio, S(stream));
    });
}

int bsml_lora_backward(bsml_lora* l, const float* daudio, void* stream) {
    return guarded([&] {
        need(l != nullptr && daudio != nullptr, "bsml_lora_backward", "null argument");
        l->lora->backward(daudio, S(stream));
    });
}

int bsml_lora_zero_grad(bsml_lora* l, void* stream) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_zero_grad", "null handle");
        l->lora->zero_grad(S(stream));
    });
}

int bsml_lora_adam_step(bsml_lora* l, float lr, float beta1, float beta2, float eps, void* stream) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_adam_step", "null handle");
        l->lora->adam_step(lr, beta1, beta2, eps, S(stream));
    });
}

int bsml_lora_save(const bsml_lora* l, const char* path) {
    return guarded([&] {
        need(l != nullptr && path != nullptr, "bsml_lora_save", "null argument");
        l->lora->save(path);
    });
}

int bsml_lora_load(bsml_lora* l, const char* path) {
    return guarded([&] {
        need(l != nullptr && path != nullptr, "bsml_lora_load", "null argument");
        l->lora->load(path);
    });
}

int bsml_lora_save_state(const bsml_lora* l, const char* path) {
    return guarded([&] {
        need(l != nullptr && path != nullptr, "bsml_lora_save_state", "null argument");
        l->lora->save(path, true);
    });
}

int bsml_lora_load_state(bsml_lora* l, const char* path) {
    return guarded([&] {
        need(l != nullptr && path != nullptr, "bsml_lora_load_state", "null argument");
        l->lora->load(path, true);
    });
}

int bsml_lora_state(const bsml_lora* l, float* scale, int* step) {
    return guarded([&] {
        need(l != nullptr, "bsml_lora_state", "null handle");
        if (scale) *scale = l->lora->scale();
        if (step) *step = l->lora->step();
    });
}

int bsml_convlora_create(bsml_decoder* d, int rank, float scale, uint64_t seed, bsml_convlora** out) {
    return guarded([&] {
        need(d && out, "bsml_convlora_create", "null argument");
        auto* l = new bsml_convlora;
        try {
            l->lora = std::make_unique<bsml::ConvLora>(*d->eng, rank, scale, seed);
        } catch (...) {
            delete l;
            throw;
        }
        *out = l;
    });
}

void bsml_convlora_destroy(bsml_convlora* l) { delete l; }

int bsml_convlora_layout(const bsml_convlora* l, int64_t* n_params, int* n_weights, int64_t* w_off, int* rows,
                         int* cols, int64_t* off_A, int64_t* off_B) {
    return guarded([&] {
        need(l != nullptr, "bsml_convlora_layout", "null handle");
        const auto& ws = l->lora->weights();
        if (n_params) *n_params = l->lora->n_params();
        if (n_weights) *n_weights = (int)ws.size();
        for (size_t i = 0; i < ws.size(); ++i) {
            if (w_off) w_off[i] = ws[i].w;
            if (rows) rows[i] = ws[i].rows;
            if (cols) cols[i] = ws[i].cols;
            if (off_A) off_A[i] = ws[i].offA;
            if (off_B) off_B[i] = ws[i].offB;
        }
    });
}

int bsml_convlora_buffers(bsml_convlora* l, float** params, float** grads) {
    return guarded([&] {
        need(l != nullptr, "bsml_convlora_buffers", "null handle");
        if (params) *params = l->lora->params();
        if (grads) *grads = l->lora->grads();
    });
}

int bsml_convlora_forward(bsml_convlora* l, int B, int T, const float* params, const float* asr, const float* F0,
                          const float* N, const float* style, const float* har, int frames, float* audio,
                          void* stream) {
    return guarded([&] {
        need(l != nullptr, "bsml_convlora_forward", "null handle");
        l->lora->forward(B, T, params, asr, F0, N, style, har, frames, audio, S(stream));
    });
}

int bsml_convlora_backward(bsml_convlora* l, const float* daudio, void* stream) {
    return guarded([&] {
        need(l != nullptr && daudio != nullptr, "bsml_convlora_backward", "null argument");
        l->lora->backward(daudio, S(stream));
    });
}

int bsml_convlora_zero_grad(bsml_convlora* l, void* stream) {
    return guarded([&] {
        need(l != nullptr, "bsml_convlora_zero_grad", "null handle");
        l->lora->zero_grad(S(stream));
    });
}

int bsml_convlora_save(const bsml_convlora* l, const char* path) {
    return guarded([&] {
        need(l != nullptr && path != nullptr, "bsml_convlora_save", "null argument");
        l->lora->save(path);
    });
}

int bsml_convlora_load(bsml_convlora* l, const char* path) {
    return guarded([&] {
        need(l != nullptr && path != nullptr, "bsml_convlora_load", "null argument");
        l->lora->load(path);
    });
}

int bsml_convlora_adam_step(bsml_convlora* l, float lr, float beta1, float beta2, float eps, void* stream) {
    return guarded([&] {
        need(l != nullptr, "bsml_convlora_adam_step", "null handle");
        l->lora->adam_step(lr, beta1, beta2, eps, S(stream));
    });
}

struct bsml_st {
    std::unique_ptr<bsml::SafeTensors> f;
};

int bsml_st_open(const char* path, bsml_st** out) {
    return guarded([&] {
        need(path && out, "bsml_st_open", "null argument");
        auto* s = new bsml_st;
        try {
            s->f = std::make_unique<bsml::SafeTensors>(path);
        } catch (...) {
            delete s;
            throw;
        }
        *out = s;
    });
}

void bsml_st_close(bsml_st* f) { delete f; }

int bsml_st_count(const bsml_st* f, int* n) {
    return guarded([&] {
        need(f && n, "bsml_st_count", "null argument");
        *n = (int)f->f->entries().size();
    });
}

int bsml_st_info(const bsml_st* f, int i, char* name, int name_cap, int* dtype, int* ndim, int64_t* shape) {
    return guarded([&] {
        need(f != nullptr, "bsml_st_info", "null handle");
        const auto& es = f->f->entries();
        need(i >= 0 && i < (int)es.size(), "bsml_st_info", "index out of range");
        const auto& e = es[i];
        if (name && name_cap > 0) {
            std::strncpy(name, e.name.c_str(), (size_t)name_cap - 1);
            name[name_cap - 1] = '\0';
        }
        if (dtype) *dtype = e.dtype;
        if (ndim) *ndim = (int)e.shape.size();
        if (shape)
            for (size_t k = 0; k < e.shape.size() && k < 8; ++k) shape[k] = e.shape[k];
    });
}

int bsml_st_read_f32(const bsml_st* f, const char* name, float* dst, int64_t n) {
    return guarded([&] {
        need(f && name && dst, "bsml_st_read_f32", "null argument");
        const auto* e = f->f->find(name);
        if (!e) bsml::fail("bsml_st_read_f32", std::string("missing safetensors key '") + name + "'");
        if (e->numel != n)
            bsml::fail("bsml_st_read_f32", std::string("tensor '") + name + "' has " + std::to_string(e->numel) +
                                               " elements; expected " + std::to_string(n));
        f->f->read_f32(*e, dst);
    });
}

int bsml_st_metadata(const bsml_st* f, const char* key, char* value, int cap) {
    return guarded([&] {
        need(f && key && value && cap > 0, "bsml_st_metadata", "null argument");
        const auto& m = f->f->metadata();
        auto it = m.find(key);
        if (it == m.end()) bsml::fail("bsml_st_metadata", std::string("no metadata key '") + key + "'");
        std::strncpy(value, it->second.c_str(), (size_t)cap - 1);
        value[cap - 1] = '\0';
    });
}

int bsml_params_from_safetensors(const bsml_st* f, const bsml_param_entry* table, int n_entries, const char* prefix,
                                 float* params, int64_t n_params) {
    return guarded([&] {
        need(f && table && params, "bsml_params_from_safetensors", "null argument");
        f->f->load_params(table, n_entries, prefix ? prefix : "", params, n_params);
    });
}

int bsml_nccl_unique_id(void* id) {
    return guarded([&] {
        need(id != nullptr, "bsml_nccl_unique_id", "null argument");
        bsml::nccl_unique_id(id);
    });
}

int bsml_nccl_comm_init_timeout(int nranks, const void* id, int rank, int device, int timeout_ms, void** comm) {
    return guarded([&] {
        need(id != nullptr && comm != nullptr, "bsml_nccl_comm_init", "null argument");
        *comm = nullptr;
        *comm = bsml::nccl_comm_init(nranks, id, rank, device, timeout_ms);
    });
}

int bsml_nccl_comm_init(int nranks, const void* id, int rank, int device, void** comm) {
    return bsml_nccl_comm_init_timeout(nranks, id, rank, device, BSML_NCCL_DEFAULT_TIMEOUT_MS, comm);
}

int bsml_nccl_comm_destroy(void* comm) {
    return guarded([&] { bsml::nccl_comm_destroy(comm); });
}

int bsml_allreduce_grads(void* comm, float* grads, int64_t n, int average, void* stream) {
    return guarded([&] { bsml::nccl_allreduce(comm, grads, n, average != 0, S(stream)); });
}

int bsml_nccl_sync(void* comm, void* stream) {
    return guarded([&] { bsml::nccl_sync(comm, S(stream)); });
}

int bsml_nccl_version(int* version) {
    return guarded([&] {
        need(version != nullptr, "bsml_nccl_version", "null argument");
        *version = bsml::nccl_version();
    });
}

struct bsml_graph {
    cudaGraph_t g = nullptr;
    cudaGraphExec_t e = nullptr;
};

int bsml_graph_begin(void* stream) {
    return guarded([&] {
        need(stream != nullptr, "bsml_graph_begin", "capture needs a stream other than the legacy default stream");
        BSML_CUDA(cudaStreamBeginCapture(S(stream), cudaStreamCaptureModeThreadLocal));
    });
}

int bsml_graph_end(void* stream, bsml_graph** out) {
    return guarded([&] {
        need(stream != nullptr && out != nullptr, "bsml_graph_end", "null argument");
        cudaGraph_t g = nullptr;
        BSML_CUDA(cudaStreamEndCapture(S(stream), &g));
        auto* G = new bsml_graph;
        G->g = g;
        const cudaError_t e = cudaGraphInstantiate(&G->e, g, 0);
        if (e != cudaSuccess) {
            cudaGraphDestroy(g);
            delete G;
            bsml::check_cuda(e, "cudaGraphInstantiate");
        }
        *out = G;
    });
}

int bsml_graph_launch(bsml_graph* g, void* stream) {
    return guarded([&] {
        need(g != nullptr, "bsml_graph_launch", "null graph");
        BSML_CUDA(cudaGraphLaunch(g->e, S(stream)));
    });
}

int bsml_graph_kernel_count(const bsml_graph* g, int64_t* n) {
    return guarded([&] {
        need(g != nullptr && n != nullptr, "bsml_graph_kernel_count", "null argument");
        size_t nn = 0;
        BSML_CUDA(cudaGraphGetNodes(g->g, nullptr, &nn));
        std::vector<cudaGraphNode_t> nodes(nn);
        if (nn) BSML_CUDA(cudaGraphGetNodes(g->g, nodes.data(), &nn));
        int64_t k = 0;
        for (auto node : nodes) {
            cudaGraphNodeType t;
            BSML_CUDA(cudaGraphNodeGetType(node, &t));
            if (t == cudaGraphNodeTypeKernel) ++k;
        }
        *n = k;
    });
}

void bsml_graph_destroy(bsml_graph* g) {
    if (!g) return;
    if (g->e) cudaGraphExecDestroy(g->e);
    if (g->g) cudaGraphDestroy(g->g);
    delete g;
}

int bsml_loss_l1(const float* audio, const float* target, int64_t n, float* loss, float* daudio, void* stream) {
    return guarded([&] {
        need(audio && target && loss && daudio && n > 0, "bsml_loss_l1", "bad argument");
        Scratch sc(S(stream));
        bsml::l1_loss(audio, target, n, loss, daudio, sc.d(1), S(stream));
    });
}

int bsml_adam_step(float* param, const float* grad, float* m, float* v, int64_t n, float lr, float beta1,
                   float beta2, float eps, int step, void* stream) {
    return guarded([&] {
        need(param && grad && m && v && step >= 1, "bsml_adam_step", "bad argument");
        bsml::adam(param, grad, m, v, n, lr, beta1, beta2, eps, step, S(stream));
    });
}

// ── atoms

int bsml_conv1d_forward(const float* x, int B, int Ci, int L, const float* W, const float* bias, int Co, int k,
                        int stride, int pad, int dil, float* y, void* stream) {
    return guarded([&] {
        const int Lo = conv_out(L, k, stride, pad, dil);
        need(x && W && y && B > 0 && Ci > 0 && Co > 0 && Lo > 0, "bsml_conv1d_forward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act xa = sc.act(B, L, Ci), ya = sc.act(B, Lo, Co);
        bsml::ncl_to_cl(x, xa, st);
        if (atom_tc(Ci, Co, stride)) {
            atom_tc_conv(sc, xa, W, bsml::PACK_CONV_FWD, Co, Ci, k, 1, 0, k, Co, ya, bias, pad, dil, Lo, 0, 1, 0, st);
        } else {
            float* wp = sc.f((int64_t)k * Ci * bsml::round_up(Co, 4));
            bsml::pack_conv_fwd(W, Co, Ci, k, wp, st);
            bsml::ConvFwd a;
            a.x = xa; a.y = ya; a.wp = wp; a.bias = bias; a.k = k; a.s = stride; a.p = pad; a.d = dil; a.No = Lo;
            bsml::conv_fwd_simt(a, st);
        }
        bsml::cl_to_ncl(ya, y, st);
    });
}

int bsml_conv1d_backward_input(const float* dy, int B, int Ci, int L, const float* W, int Co, int k, int stride,
                               int pad, int dil, float* dx, void* stream) {
    return guarded([&] {
        need(stride == 1, "bsml_conv1d_backward_input", "only stride 1 is supported");
        const int Lo = conv_out(L, k, stride, pad, dil);
        need(dy && W && dx && B > 0 && Lo > 0, "bsml_conv1d_backward_input", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act ga = sc.act(B, Lo, Co), xa = sc.act(B, L, Ci);
        bsml::ncl_to_cl(dy, ga, st);
        if (atom_tc(Co, Ci, 1)) {
            atom_tc_conv(sc, ga, W, bsml::PACK_CONV_DGRAD, Co, Ci, k, 1, 0, k, Ci, xa, nullptr, dil * (k - 1) - pad, dil,
                         L, 0, 1, 0, st, atom_dg_mode());
        } else {
            float* wp = sc.f((int64_t)k * Co * bsml::round_up(Ci, 4));
            bsml::pack_conv_dgrad(W, Co, Ci, k, wp, st);
            bsml::ConvFwd a;
            a.x = ga; a.y = xa; a.wp = wp; a.k = k; a.s = 1; a.p = dil * (k - 1) - pad; a.d = dil; a.No = L;
            bsml::conv_fwd_simt(a, st);
        }
        bsml::cl_to_ncl(xa, dx, st);
    });
}

int bsml_conv1d_backward_weight(const float* dy, const float* x, int B, int Ci, int L, int Co, int k, int stride,
                                int pad, int dil, float* dW, float* db, void* stream) {
    return guarded([&] {
        const int Lo = conv_out(L, k, stride, pad, dil);
        need(dy && x && dW && B > 0 && Lo > 0, "bsml_conv1d_backward_weight", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act ga = sc.act(B, Lo, Co), xa = sc.act(B, L, Ci);
        bsml::ncl_to_cl(dy, ga, st);
        bsml::ncl_to_cl(x, xa, st);
        if (atom_tc(Ci, Co, stride)) {
            const int mode = atom_wg_mode();
            float* yh = sc.f((int64_t)B * Lo * bsml::tc_pitch(Co, mode));
            float* yl = sc.f((int64_t)B * Lo * bsml::tc_pitch(Co, mode));
            float* xh = sc.f((int64_t)B * L * bsml::tc_pitch(Ci, mode));
            float* xl = sc.f((int64_t)B * L * bsml::tc_pitch(Ci, mode));
            bsml::make_act_planes(ga, mode, yh, yl, st);
            bsml::make_act_planes(xa, mode, xh, xl, st);
            bsml::TcConvWgrad w;
            w.dy.hi = yh; w.dy.lo = yl; w.dy.ld = bsml::tc_pitch(Co, mode);
            w.x.hi = xh; w.x.lo = xl; w.x.ld = bsml::tc_pitch(Ci, mode);
            w.B = B; w.Lo = Lo; w.Co = Co; w.L_in = L; w.Ci = Ci; w.taps = k; w.p = pad; w.d = dil; w.dW = dW;
            const int64_t cap = std::max<int64_t>(std::min<int64_t>(48ll << 20, 296ll * Co * Ci * k),
                                                  bsml::colsum_partial_floats(ga));
            float* part = sc.f(cap);
            bsml::conv_wgrad_tc(w, mode, part, cap, st);
            if (db) bsml::colsum(ga, db, false, part, st);
            return;
        }
        bsml::ConvWgrad a;
        a.dy = ga; a.x = xa; a.k = k; a.s = stride; a.p = pad; a.d = dil; a.dW = dW; a.db = db;
        float* part = sc.f(std::max(bsml::wgrad_partial_floats(a), bsml::colsum_partial_floats(ga)));
        bsml::conv_wgrad_simt(a, part, st);
    });
}

int bsml_conv_transpose1d_forward(const float* x, int B, int Ci, int L, const float* W, const float* bias, int Co,
                                  int k, int stride, int pad, float* y, void* stream) {
    return guarded([&] {
        const int Lu = (L - 1) * stride - 2 * pad + k;
        need(x && W && y && B > 0 && Lu > 0, "bsml_conv_transpose1d_forward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act xa = sc.act(B, L, Ci), ya = sc.act(B, Lu, Co);
        bsml::ncl_to_cl(x, xa, st);
        for (int ph = 0; ph < stride; ++ph) {
            const int kr = (k - ph + stride - 1) / stride;
            if (kr <= 0) continue;
            const int qmin = (int)bsml::ceil_div(std::max(pad - ph, 0), stride);
            const int qmax = (Lu - 1 + pad - ph) >= 0 ? (Lu - 1 + pad - ph) / stride : -1;
            if (qmax < qmin) continue;
            if (atom_tc(Ci, Co, 1)) {
                atom_tc_conv(sc, xa, W, bsml::PACK_CONVT_PHASE, Co, Ci, k, stride, ph, kr, Co, ya, bias, kr - 1, 1,
                             qmax - qmin + 1, qmin, stride, ph - pad, st);
                continue;
            }
            float* wp = sc.f((int64_t)kr * Ci * bsml::round_up(Co, 4));
            bsml::pack_convT_phase(W, Ci, Co, k, stride, ph, wp, st);
            bsml::ConvFwd a;
            a.x = xa; a.y = ya; a.wp = wp; a.bias = bias; a.k = kr; a.s = 1; a.p = kr - 1; a.d = 1;
            a.No = qmax - qmin + 1; a.o_base = qmin; a.orow_mul = stride; a.orow_off = ph - pad;
            bsml::conv_fwd_simt(a, st);
        }
        bsml::cl_to_ncl(ya, y, st);
    });
}

int bsml_conv_transpose1d_backward_input(const float* dy, int B, int Ci, int L, const float* W, int Co, int k,
                                         int stride, int pad, float* dx, void* stream) {
    return guarded([&] {
        const int Lu = (L - 1) * stride - 2 * pad + k;
        need(dy && W && dx && B > 0 && Lu > 0, "bsml_conv_transpose1d_backward_input", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act ga = sc.act(B, Lu, Co), xa = sc.act(B, L, Ci);
        bsml::ncl_to_cl(dy, ga, st);
        if (atom_convT_tc(Ci, Co, stride, Lu)) {
            const int mode = atom_dg_mode();
            const bsml::ConvTPack pk = bsml::convT_pack(k, stride, pad);
            const int K = stride * Co;
            float* gh = sc.f((int64_t)B * Lu * Co);
            float* gl = sc.f((int64_t)B * Lu * Co);
            const int64_t wn = (int64_t)pk.taps * Ci * bsml::round_up(K, 8);
            float* wh = sc.f(wn);
            float* wl = sc.f(wn);
            bsml::make_act_planes(ga, mode, gh, gl, st);
            bsml::pack_w_tc(W, bsml::PACK_CONVT_DGRAD, Co, Ci, k, stride, pad, mode, wh, wl, st);
            bsml::TcConvFwd a;
            a.x.hi = gh; a.x.lo = gl; a.x.ld = K;
            a.B = B; a.L_in = Lu / stride; a.Ci = K;
            a.w.hi = wh; a.w.lo = wl; a.w.ld = (int)bsml::round_up(K, 8);
            a.taps = pk.taps; a.Co = Ci; a.p = -pk.u_min; a.d = 1; a.No = L;
            a.y = xa;
            a.part_cap = bsml::conv_fwd_tc_part_floats(a, mode);
            if (a.part_cap > 0) a.part = sc.f(a.part_cap);
            bsml::conv_fwd_tc(a, mode, st);
            bsml::cl_to_ncl(xa, dx, st);
            return;
        }
        float* wp = sc.f((int64_t)k * Co * bsml::round_up(Ci, 4));
        bsml::pack_convT_dgrad(W, Ci, Co, k, wp, st);
        bsml::ConvFwd a;
        a.x = ga; a.y = xa; a.wp = wp; a.k = k; a.s = stride; a.p = pad; a.d = 1; a.No = L;
        bsml::conv_fwd_simt(a, st);
        bsml::cl_to_ncl(xa, dx, st);
    });
}

int bsml_conv_transpose1d_backward_weight(const float* dy, const float* x, int B, int Ci, int L, int Co, int k,
                                          int stride, int pad, float* dW, float* db, void* stream) {
    return guarded([&] {
        const int Lu = (L - 1) * stride - 2 * pad + k;
        need(dy && x && dW && B > 0 && Lu > 0, "bsml_conv_transpose1d_backward_weight", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act ga = sc.act(B, Lu, Co), xa = sc.act(B, L, Ci);
        bsml::ncl_to_cl(dy, ga, st);
        bsml::ncl_to_cl(x, xa, st);
        if (atom_convT_tc(Ci, Co, stride, Lu)) {
            const int mode = atom_wg_mode();
            const bsml::ConvTPack pk = bsml::convT_pack(k, stride, pad);
            const int K = stride * Co;
            float* gh = sc.f((int64_t)B * Lu * Co);
            float* gl = sc.f((int64_t)B * Lu * Co);
            float* xh = sc.f((int64_t)B * L * bsml::tc_pitch(Ci, mode));
            float* xl = sc.f((int64_t)B * L * bsml::tc_pitch(Ci, mode));
            bsml::make_act_planes(ga, mode, gh, gl, st);
            bsml::make_act_planes(xa, mode, xh, xl, st);
            bsml::TcConvWgrad w;
            w.dy.hi = xh; w.dy.lo = xl; w.dy.ld = bsml::tc_pitch(Ci, mode);
            w.x.hi = gh; w.x.lo = gl; w.x.ld = K;
            w.B = B; w.Lo = L; w.Co = Ci; w.L_in = Lu / stride; w.Ci = K;
            w.taps = pk.taps; w.p = -pk.u_min; w.d = 1; w.dW = dW;
            w.ct_s = stride; w.ct_p = pad; w.ct_k = k; w.ct_Co = Co;
            const int64_t cap = std::max<int64_t>(std::min<int64_t>(48ll << 20, 296ll * Ci * K * pk.taps),
                                                  bsml::colsum_partial_floats(ga));
            float* part = sc.f(cap);
            bsml::conv_wgrad_tc(w, mode, part, cap, st);
            if (db) bsml::colsum(ga, db, false, part, st);
            return;
        }
        bsml::ConvWgrad a;
        a.dy = xa; a.x = ga; a.k = k; a.s = stride; a.p = pad; a.d = 1; a.dW = dW;
        float* part = sc.f(std::max(bsml::wgrad_partial_floats(a), bsml::colsum_partial_floats(ga)));
        bsml::conv_wgrad_simt(a, part, st);
        if (db) bsml::colsum(ga, db, false, part, st);
    });
}

int bsml_adain_affine_forward(const float* x, const float* gb, int B, int C, int L, float eps, float* y,
                              void* stream) {
    return guarded([&] {
        need(x && gb && y && B > 0 && C > 0 && L > 0, "bsml_adain_affine_forward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act xa = sc.act(B, L, C), ya = sc.act(B, L, C);
        float* mean = sc.f((int64_t)B * C);
        float* rstd = sc.f((int64_t)B * C);
        bsml::ncl_to_cl(x, xa, st);
        bsml::in_stats(xa, eps, sc.d((int64_t)B * C * 2), mean, rstd, st);
        bsml::adain_act_fwd(xa, mean, rstd, gb, bsml::ACT_NONE, 0.f, nullptr, ya, st);
        bsml::cl_to_ncl(ya, y, st);
    });
}

int bsml_adain_affine_backward(const float* x, const float* gb, const float* dy, int B, int C, int L, float eps,
                               float* dx, float* dgb, void* stream) {
    return guarded([&] {
        need(x && gb && dy && dx && dgb && B > 0 && C > 0 && L > 0, "bsml_adain_affine_backward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act xa = sc.act(B, L, C), ga = sc.act(B, L, C), da = sc.act(B, L, C);
        float* mean = sc.f((int64_t)B * C);
        float* rstd = sc.f((int64_t)B * C);
        double* acc = sc.d((int64_t)B * C * 3);
        bsml::ncl_to_cl(x, xa, st);
        bsml::ncl_to_cl(dy, ga, st);
        bsml::in_stats(xa, eps, acc, mean, rstd, st);
        bsml::adain_act_bwd(xa, mean, rstd, gb, bsml::ACT_NONE, 0.f, nullptr, ga, da, nullptr, dgb, nullptr, acc, st);
        bsml::cl_to_ncl(da, dx, st);
    });
}

int bsml_snake_forward(const float* x, const float* alpha, int B, int C, int L, float* y, void* stream) {
    return guarded([&] {
        need(x && alpha && y && B > 0 && C > 0 && L > 0, "bsml_snake_forward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act xa = sc.act(B, L, C), ya = sc.act(B, L, C);
        bsml::ncl_to_cl(x, xa, st);
        bsml::snake_fwd(xa, alpha, ya, st);
        bsml::cl_to_ncl(ya, y, st);
    });
}

int bsml_snake_backward(const float* x, const float* alpha, const float* dy, int B, int C, int L, float* dx,
                        float* dalpha, void* stream) {
    return guarded([&] {
        need(x && alpha && dy && dx && dalpha && B > 0 && C > 0 && L > 0, "bsml_snake_backward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::Act xa = sc.act(B, L, C), ga = sc.act(B, L, C), da = sc.act(B, L, C);
        bsml::ncl_to_cl(x, xa, st);
        bsml::ncl_to_cl(dy, ga, st);
        bsml::snake_bwd(xa, alpha, ga, da, dalpha, sc.d((int64_t)B * C), st);
        bsml::cl_to_ncl(da, dx, st);
    });
}

int bsml_istft_forward(const float* re, const float* im, int B, int n_fft, int hop, int L, float* audio,
                       void* stream) {
    return guarded([&] {
        need(re && im && audio && B > 0 && L > 1 && hop > 0, "bsml_istft_forward", "bad argument");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        bsml::istft_fwd_ncl(re, im, B, L, n_fft, hop, audio, sc.f((int64_t)B * L * (n_fft + 2)), st);
    });
}

int bsml_istft_backward(const float* daudio, int B, int n_fft, int hop, int L, float* dre, float* dim, void* stream) {
    return guarded([&] {
        need(daudio && dre && dim && B > 0 && L > 1 && hop > 0, "bsml_istft_backward", "bad argument");
        bsml::istft_bwd_ncl(daudio, B, L, n_fft, hop, dre, dim, S(stream));
    });
}

int bsml_spectral_head_forward(const float* x, int B, int C, int L, const float* W, const float* bias, int n_fft,
                               int hop, int post_kernel, float* post, float* audio, void* stream) {
    return guarded([&] {
        const char* where = "bsml_spectral_head_forward";
        need(x && W && post && audio && B > 0 && C > 0 && L > 1 && hop > 0, where, "bad argument");
        need(n_fft >= 2 && n_fft <= 64 && !(n_fft & 1), where, "n_fft must be even and at most 64");
        need(post_kernel >= 1 && (post_kernel & 1), where, "post_kernel must be odd");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        const int Cp = n_fft + 2, nf = n_fft / 2 + 1;
        bsml::Act xa = sc.act(B, L, C), xl = sc.act(B, L, C);
        bsml::ncl_to_cl(x, xa, st);
        bsml::leaky_fwd(xa, 0.01f, xl, st);
        // conv_post (kokoro_decoder_backward.cpp:387-389) through the conv atom (NCL)
        float* xl_ncl = sc.f((int64_t)B * C * L);
        bsml::cl_to_ncl(xl, xl_ncl, st);
        check_rc(bsml_conv1d_forward(xl_ncl, B, C, L, W, bias, Cp, post_kernel, 1, (post_kernel - 1) / 2, 1, post,
                                     stream));
        bsml::Act pa = sc.act(B, L, Cp);
        bsml::ncl_to_cl(post, pa, st);
        float* spec = sc.f((int64_t)B * L * 2 * nf);
        bsml::polar_fwd(pa, nf, spec, st);
        bsml::istft_fwd(spec, B, L, n_fft, hop, audio, st);
    });
}

int bsml_spectral_head_backward(const float* x, const float* post, const float* daudio, int B, int C, int L,
                                const float* W, int n_fft, int hop, int post_kernel, float* dx, void* stream) {
    return guarded([&] {
        const char* where = "bsml_spectral_head_backward";
        need(x && post && daudio && W && dx && B > 0 && C > 0 && L > 1 && hop > 0, where, "bad argument");
        need(n_fft >= 2 && n_fft <= 64 && !(n_fft & 1), where, "n_fft must be even and at most 64");
        need(post_kernel >= 1 && (post_kernel & 1), where, "post_kernel must be odd");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        const int Cp = n_fft + 2;
        bsml::Act pa = sc.act(B, L, Cp), dpa = sc.act(B, L, Cp);
        bsml::ncl_to_cl(post, pa, st);
        // iSTFT adjoint fused with the polar exp / sin adjoint (kokoro_decoder_backward.cpp:424-451)
        bsml::istft_polar_bwd(daudio, pa, n_fft, hop, dpa, st);
        float* dpost = sc.f((int64_t)B * Cp * L);
        bsml::cl_to_ncl(dpa, dpost, st);
        float* dxl = sc.f((int64_t)B * C * L);
        check_rc(bsml_conv1d_backward_input(dpost, B, C, L, W, Cp, post_kernel, 1, (post_kernel - 1) / 2, 1, dxl,
                                            stream));
        bsml::Act xa = sc.act(B, L, C), dxla = sc.act(B, L, C), dxa = sc.act(B, L, C);
        bsml::ncl_to_cl(x, xa, st);
        bsml::ncl_to_cl(dxl, dxla, st);
        bsml::leaky_bwd(xa, 0.01f, dxla, dxa, st);
        bsml::cl_to_ncl(dxa, dx, st);
    });
}

int bsml_transpose(const float* src, int64_t batch, int rows, int cols, float* dst, void* stream) {
    return guarded([&] {
        need(src && dst && batch > 0 && rows > 0 && cols > 0, "bsml_transpose", "bad argument");
        // (batch, rows, cols) -> (batch, cols, rows): the channels-last conversion with C = rows
        cudaStream_t st = S(stream);
        bsml::Act a;
        a.B = (int)batch; a.L = cols; a.C = rows; a.ld = rows; a.bstride = (int64_t)rows * cols;
        a.p = dst;
        bsml::ncl_to_cl(src, a, st);
    });
}

int bsml_managed_alloc(int64_t bytes, void** out) {
    return guarded([&] {
        need(out != nullptr && bytes >= 0, "bsml_managed_alloc", "bad argument");
        *out = nullptr;
        void* p = nullptr;
        bsml::check_cuda(cudaMallocManaged(&p, std::max<int64_t>(bytes, 16)), "cudaMallocManaged");
        bsml::check_cuda(cudaMemset(p, 0, std::max<int64_t>(bytes, 16)), "cudaMemset");
        bsml::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        *out = p;
    });
}

int bsml_managed_free(void* p) {
    return guarded([&] {
        if (p) bsml::check_cuda(cudaFree(p), "cudaFree");
    });
}

int bsml_synchronize(void) {
    return guarded([&] { bsml::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); });
}

int bsml_memcpy(void* dst, const void* src, int64_t bytes, void* stream) {
    return guarded([&] {
        need(dst && src && bytes >= 0, "bsml_memcpy", "bad argument");
        bsml::check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, S(stream)), "cudaMemcpyAsync");
    });
}

int bsml_harmonic_source_mode(const bsml_decoder_config* cfg, const float* F0, int B, int F, const float* l_weight,
                              const float* l_bias, float* har, int phase_mode, void* stream) {
    return guarded([&] {
        need(cfg && F0 && l_weight && l_bias && har && B > 0 && F > 0, "bsml_harmonic_source", "bad argument");
        need(phase_mode == BSML_PHASE_FP32_RUNNING || phase_mode == BSML_PHASE_EXACT, "bsml_harmonic_source",
             "unknown phase mode");
        cudaStream_t st = S(stream);
        Scratch sc(st);
        const int S_len = F * cfg->upsample_scale;
        const int frames = S_len / cfg->hop + 1;
        bsml::Act ha = sc.act(B, frames, cfg->n_fft + 2);
        bsml::harmonic_source(F0, B, F, cfg->upsample_scale, cfg->harmonic_num, cfg->sample_rate, cfg->n_fft, cfg->hop,
                              l_weight, l_bias, sc.d((int64_t)B * (cfg->harmonic_num + 1) * F), sc.f((int64_t)B * S_len),
                              ha, st, phase_mode);
        bsml::cl_to_ncl(ha, har, st);
    });
}

int bsml_harmonic_source(const bsml_decoder_config* cfg, const float* F0, int B, int F, const float* l_weight,
                         const float* l_bias, float* har, void* stream) {
    return bsml_harmonic_source_mode(cfg, F0, B, F, l_weight, l_bias, har, BSML_PHASE_FP32_RUNNING, stream);
}

int bsml_decoder_set_phase_mode(bsml_decoder* d, int phase_mode) {
    return guarded([&] {
        need(d != nullptr, "bsml_decoder_set_phase_mode", "null handle");
        d->eng->set_phase_mode(phase_mode);
    });
}

}  // extern "C"
