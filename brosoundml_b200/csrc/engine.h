// The batched decoder engine: forward with caches, backward, workspace planning.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <vector>

#include "common.cuh"
#include "conv_tc.h"
#include "kernels.h"
#include "layout.h"

namespace bsml {

class Engine {
   public:
    Engine(const bsml_decoder_config& cfg, int device);
    Engine(const bsml_block_spec& spec, int device);   // one block on its own
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    const Layout& layout() const { return lay_; }
    void set_math(int m);
    int math() const { return math_; }

    // style rows are style_stride floats apart (0 = style_dim; a (B, 2*style_dim)
    // ref_s passes 2*style_dim and the decoder reads the first style_dim of each row)
    void forward(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                 const float* style, const float* har, int frames, const float* aff_in, float* audio,
                 float* aff_out, cudaStream_t st, int style_stride = 0);
    void backward(const float* daudio, float* grads, float* d_asr, float* d_style, float* d_aff, cudaStream_t st);
    // The two assemblies on their own (detail::decoder_backbone_* / generator_*,
    // src/kokoro_decoder_backward.h:213-293): the backbone maps (asr, F0, N) to
    // gen_in (B, init_ch, L_gen) NCL; the generator maps gen_in (B, init_ch, L_in)
    // and har (B, har_ch, frames) to audio. Affines: the whole packing, of which
    // each part reads (and writes the gradients of) its own AdaINs.
    void forward_backbone(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                          const float* style, int style_stride, const float* aff_in, float* gen_in, float* aff_out,
                          cudaStream_t st);
    void backward_backbone(const float* dgen_in, float* grads, float* d_asr, float* d_style, float* d_aff,
                           cudaStream_t st);
    void forward_generator(int B, int L_in, const float* params, const float* gen_in, const float* har, int frames,
                           const float* style, int style_stride, const float* aff_in, float* audio, float* aff_out,
                           cudaStream_t st);
    void backward_generator(const float* daudio, float* grads, float* dgen_in, float* d_style, float* d_aff,
                            cudaStream_t st);
    // gen_in length of the backbone for T asr frames
    int backbone_out_len(int T) const;
    // one block (a handle made from a bsml_block_spec): x, y, dy, dx NCL
    void forward_block(int B, int L, const float* params, const float* x, const float* style, const float* aff_in,
                       float* y, float* aff_out, cudaStream_t st);
    void backward_block(const float* dy, float* grads, float* dx, float* d_style, float* d_aff, cudaStream_t st);
    int64_t workspace_bytes() const { return ws_bytes_ + wp_bytes_ + tcw_bytes_; }

    // Per-kernel-class timing with CUDA events (off by default); the classes of
    // bsml_decoder_read_profile. Per class: ms, algorithmic work (FLOPs for the
    // convs, bytes for the norms), launches. Reading synchronises the device.
    enum {
        PROF_CONV_TC = BSML_PROF_CONV_TC, PROF_CONV_SIMT = BSML_PROF_CONV_SIMT, PROF_WGRAD_TC = BSML_PROF_WGRAD_TC,
        PROF_WGRAD_SIMT = BSML_PROF_WGRAD_SIMT, PROF_NORM_FWD = BSML_PROF_NORM_FWD,
        PROF_NORM_BWD = BSML_PROF_NORM_BWD, PROF_N = BSML_PROF_CLASSES
    };
    void set_profiling(bool on);
    // harmonic-source phase arithmetic: PHASE_FP32_RUNNING (the reference's, default) or PHASE_EXACT
    void set_phase_mode(int m);
    void read_profile(double* out);   // PROF_N * 3 doubles, then clears
    // per launch in issue order: (class, work, ms), at most max_records; then clears
    void read_profile_records(double* out, int max_records, int* n_records);

   private:
    // ── planning
    struct Planner {
        char* base = nullptr;
        int64_t off = 0;
        void* take(int64_t bytes) {
            off = round_up(off, 256);
            void* p = base ? base + off : nullptr;
            off += bytes;
            return p;
        }
        Act act(int B, int L, int C) {
            Act a;
            a.B = B; a.L = L; a.C = C; a.ld = pitch(C);
            a.bstride = (int64_t)L * a.ld;
            a.p = (float*)take((int64_t)B * a.bstride * 4);
            return a;
        }
        float* f(int64_t n) { return (float*)take(n * 4); }
        double* d(int64_t n) { return (double*)take(n * 8); }
    };
    struct Stats { float* mean = nullptr; float* rstd = nullptr; };
    struct BlkC { Act x, r, pooled, c1, n2, sc; Stats s1, s2; int Lin = 0, Lout = 0; };
    // AdaINResBlock1 caches: block inputs x[i] and conv1 outputs c1[i] with
    // their statistics. The Snake outputs are not kept: the backward recomputes
    // them from x[i] / c1[i] and the statistics.
    struct RB1C { Act x[3], c1[3]; Stats st1[3], st2[3]; int L = 0; };
    struct StageC { Act x_in, a, xsrc, src, m, out; RB1C noise; std::vector<RB1C> res; int Lin = 0, Lu = 0, Lx = 0; };

    void init();
    void plan(Planner& P);
    void plan_block(Planner& P);
    void plan_scratch(Planner& P, int64_t max_elems, int max_c);
    enum { PART_FULL = 0, PART_BACKBONE = 1, PART_GENERATOR = 2 };
    void ensure_plan(int B, int T, int frames, bool have_har, int part);
    void begin_forward(int B, int T, int frames, bool have_har, int part, const float* params, const float* F0,
                       const float* N, const float* style, int style_stride, const float* aff_in, float* aff_out,
                       cudaStream_t st);
    void run_backbone(const float* asr, cudaStream_t st);
    void run_generator(const float* har, float* audio, cudaStream_t st);
    void begin_backward(const char* where, int part, float* grads, cudaStream_t st);
    Act gen_backward(const float* daudio, cudaStream_t st);
    void bb_backward(Act dY, cudaStream_t st);
    void finish_backward(float* d_style, float* d_aff, cudaStream_t st);
    Stats stats(Planner& P, int B, int C);
    BlkC plan_blk(Planner& P, const BlkP& w, int Lin, bool input_owned);
    RB1C plan_rb1(Planner& P, int L, int C);

    // ── execution helpers
    void build_pack_jobs();
    void pack_weights(cudaStream_t st);
    void pack_dgrad_weights(cudaStream_t st);
    const float* aff(const AdaP& a) const { return aff_ + (int64_t)B_ * lay_.aff_base[a.idx]; }
    float* daff(const AdaP& a) const { return daff_ + (int64_t)B_ * lay_.aff_base[a.idx]; }
    const float* P(int64_t off) const { return off >= 0 ? params_ + off : nullptr; }
    float* G(int64_t off) const { return (grads_ && off >= 0) ? grads_ + off : nullptr; }

    // A conv operand: the fp32 channels-last view (p may be null when only
    // planes exist; the geometry is always set) and / or tensor-core planes.
    struct Opnd {
        Act f;
        TcPlanes tp;
        TcPlanes tpw;   // the weight gradients' planes when their mode differs (wg_split), else unset
        const TcPlanes* planes() const { return tp.hi ? &tp : nullptr; }
        const TcPlanes* planes_w() const { return tpw.hi ? &tpw : planes(); }
    };
    // Output buffer for an elementwise producer feeding a conv: operand planes
    // (hi, lo) when that conv runs on the tensor cores, else fp32 in fbuf.
    Opnd operand(bool tc, int L, int C, const Act& fbuf, void* hi, void* lo, int mode = -1) const;
    void adain_fwd_to(const Act& x, const double* sums, const Stats& s, const float* gb, int act, float slope,
                      const float* alpha, const Opnd& out, cudaStream_t st);
    // acc_ready: the reduction pass already ran (recompute_reduce_to with the same x, dy)
    // out = gradient + skip_scale * skip (+ the prior out.f with out_accum)
    void adain_bwd_to(const Act& x, const Stats& s, const float* gb, int act, float slope, const float* alpha,
                      const Act& dy, const Opnd& out, const Act* skip, double* colsum, float* dgb, float* dalpha,
                      cudaStream_t st, bool acc_ready = false, float skip_scale = 1.f, bool out_accum = false);
    // out = act(AdaIN(x)) again, fused with the backward's reduction over (x, dy); the
    // output is a weight gradient's operand, so its planes are in wg_mode()
    void recompute_reduce_to(const Act& x, const Stats& s, const float* gb, int act, float slope, const float* alpha,
                             const Act& dy, const Opnd& out, cudaStream_t st);

    // Conv wrappers. xp / dyp: the operand's planes when a producer already
    // wrote them. stats: per-(b, co) sums of the output for the next norm
    // (zeroed here). bias_sum: the bias gradient as per-channel double sums
    // from the producer of dy (else it is summed from dy here).
    void conv(const ConvP& c, const Act& x, const Act& y, const Act* r, int r_shift, float alpha, bool accum,
              cudaStream_t st, const TcPlanes* xp = nullptr, double* stats = nullptr);
    void conv_dgrad(const ConvP& c, const Act& dy, const Act& dx, bool accum, cudaStream_t st,
                    const TcPlanes* dyp = nullptr);
    void conv_wgrad(const ConvP& c, const Act& dy, const Act& x, cudaStream_t st, const TcPlanes* dyp = nullptr,
                    const TcPlanes* xp = nullptr, const double* bias_sum = nullptr);
    void convT(const UpP& u, const Act& x, const Act& y, int row_off, const Act* r, cudaStream_t st);
    // dyp: row-packed planes of dy from convT_dy_planes (tensor cores), else CUDA cores
    void convT_dgrad(const UpP& u, const Act& dy, const Act& dx, cudaStream_t st, const TcPlanes* dyp = nullptr);
    void convT_wgrad(const UpP& u, const Act& dy, const Act& x, cudaStream_t st, const TcPlanes* dyp = nullptr);
    const TcPlanes* convT_dy_planes(const UpP& u, const Act& dy, TcPlanes& tp, cudaStream_t st);
    // ConvTranspose1d gradients on the tensor cores (row-packed form; needs Lu % s == 0 at run time)
    bool convT_tc(const UpP& u) const {
        return math_ != BSML_MATH_FP32_SIMT && u.cin >= 64 && u.s * u.cout >= 32 && u.cout % 8 == 0;
    }
    void stats_of(const Act& x, const Stats& s, cudaStream_t st);

    void blk_fwd(const BlkP& w, BlkC& c, const Act& y, cudaStream_t st);
    void blk_bwd(const BlkP& w, BlkC& c, const Act& dY, const Act& dX, cudaStream_t st);
    // x0_stats: the statistics of x0 are already in c.st1[0] (shared by the
    // resblocks of one stage, which all read the same input)
    void rb1_fwd(const RB1P& w, RB1C& c, const Act& x0, bool x0_stats, const Act& out, float out_alpha,
                 bool out_accum, cudaStream_t st);
    // Entry and exit of an AdaINResBlock1 backward inside a generator stage, whose
    // resblocks all start from the same scale * dOut and whose input gradients are
    // summed: the entry's operand planes and column sums of scale * dOut are made
    // once for the stage (the first pair reads dOut itself, scaled, as its skip
    // term), and each resblock's last pass adds its input gradient into the stage
    // sum, the last one also writing that sum's planes and column sums.
    struct RB1Io {
        const TcPlanes* in_planes = nullptr;   // planes of scale * dOut (tensor-core path)
        const TcPlanes* in_planes_w = nullptr; // the same in wg_mode (wg_split only)
        const double* in_bsum = nullptr;       // column sums of scale * dOut (nullable)
        const Act* out = nullptr;              // destination of the input gradient instead of D
        bool out_accum = false;                // out += instead of out =
        TcPlanes out_planes;                   // planes of the final out (hi null: none)
        TcPlanes out_planes_w;                 // the same in wg_mode (wg_split only)
        double* out_bsum = nullptr;            // column sums of the final out (zeroed here; nullable)
    };
    // returns the gradient w.r.t. the block input in `D` (scratch, may alias nothing
    // else), or in io->out
    void rb1_bwd(const RB1P& w, RB1C& c, const Act& dOut, float scale, const Act& D, cudaStream_t st,
                 const RB1Io* io = nullptr);

    struct ProfRec { int cls; double work; cudaEvent_t a, b; };
    int prof_begin(int cls, double work, cudaStream_t st);
    void prof_end(int id, cudaStream_t st);
    bool prof_on_ = false;
    std::vector<ProfRec> prof_;
    std::vector<cudaEvent_t> ev_pool_;
    size_t ev_used_ = 0;

    Layout lay_;
    int device_ = 0;
    int phase_mode_ = PHASE_FP32_RUNNING;
    cudaStream_t side_ = nullptr;     // harmonic source, forked from and joined to the caller's stream
    cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;
    int math_ = BSML_MATH_FP32_SIMT;

    // packed weights (persistent, independent of B/T)
    char* wp_mem_ = nullptr;
    int64_t wp_bytes_ = 0;
    std::vector<float*> wp_fwd_, wp_dgrad_;       // per conv id
    std::vector<std::vector<float*>> wp_up_;      // per ups: phases
    std::vector<float*> wp_up_dgrad_;
    // tensor-core weight planes (hi, lo) per conv id, per convT phase
    char* tcw_mem_ = nullptr;
    int64_t tcw_bytes_ = 0;
    std::vector<float*> tcw_fwd_hi_, tcw_fwd_lo_, tcw_dg_hi_, tcw_dg_lo_;
    std::vector<std::vector<float*>> tcw_up_hi_, tcw_up_lo_;
    std::vector<float*> tcw_updg_hi_, tcw_updg_lo_;   // convT input gradient, row-packed
    float* tc_xh_ = nullptr;          // activation planes of the current tensor-core call
    float* tc_xl_ = nullptr;
    float* tc_yh_ = nullptr;          // second operand's planes (weight gradients)
    float* tc_yl_ = nullptr;
    float* tc_dh_ = nullptr;          // planes of the running resblock input gradient
    float* tc_dl_ = nullptr;
    float* tc_eh_ = nullptr;          // planes of a generator stage's resblock entry gradient
    float* tc_el_ = nullptr;
    // wg_split: the weight gradients' copies of the running input gradient (tc_dh_),
    // of conv1's output gradient in a resblock pair and of the stage entry (tc_eh_)
    float* tc_dwh_ = nullptr;
    float* tc_dwl_ = nullptr;
    float* tc_uwh_ = nullptr;
    float* tc_uwl_ = nullptr;
    float* tc_ewh_ = nullptr;
    float* tc_ewl_ = nullptr;
    int tc_mode() const {
        return math_ == BSML_MATH_BF16 ? TC_BF16 : math_ == BSML_MATH_BF16X3 ? TC_BF16X3 : TC_TF32X3;
    }
    // tc_mode(): the forward's contractions and operand planes. bw_mode(): the
    // backward's input gradients and the planes its producers write (BF16X3 under
    // TF32X3F). wg_mode(): the weight gradients (BF16X3 under TF32X3W and TF32X3F:
    // their rounding ends in dW and propagates nowhere). wg_split: the last two differ
    // (TF32X3W), so an operand shared by an input and a weight gradient is written in
    // both forms.
    int bw_mode() const { return math_ == BSML_MATH_TF32X3F ? TC_BF16X3 : tc_mode(); }
    int wg_mode() const {
        return (math_ == BSML_MATH_TF32X3W || math_ == BSML_MATH_TF32X3F) ? TC_BF16X3 : tc_mode();
    }
    bool wg_split() const { return wg_mode() != bw_mode(); }
    // planes of an operand that also has fp32 data, handed to a weight gradient: under
    // wg_split the weight gradient makes its own from the fp32 data
    const TcPlanes* wgp(const TcPlanes* p) const { return wg_split() ? nullptr : p; }
    // stride-1 convs run on the tensor cores; narrow channel counts (conv_post's 22
    // outputs, the 22 harmonic channels) are zero-padded to the tile by TMA
    bool tc_ok(int K, int M, int s) const { return math_ != BSML_MATH_FP32_SIMT && s == 1 && K >= 8 && M >= 16; }
    // A strided noise conv (Kokoro: 22 -> 256, k12, stride 6) runs on the tensor cores
    // in row-packed form: the har buffer holds p zero rows before the first frame and
    // zero rows after the last, so s consecutive rows read as one row of s*ld channels
    // form a stride-1 conv with ceil(k/s) taps over K = s*ld (weights packed to match,
    // PACK_CONV_STRIDED); its weight gradient is unpacked from that form.
    // The forward runs in this form in the BF16 modes only. Under TF32x3 its result is
    // accurate per element (5.8e-7 rel-L2 against the CUDA-core conv at the bench shape)
    // but its magnitude is about 4e-7 smaller (sum of squares 8.8e-7 below the CUDA-core
    // one; consistent with the in-TMEM accumulation rounding toward zero), and the
    // decoder's gradients are ill-conditioned in that scale: scaling this conv's output
    // by 1 - 3.5e-6 moves the float64 reference's whole gradient by 1.5e-3 (the output
    // enters the stage through the noise resblock's residual path, unnormalised). It
    // took the config-2 gradient error from 1.7e-5 to 3.2e-4, past the 1e-4 bar, so
    // under TF32x3 the forward stays on the CUDA cores. The weight gradient runs in this
    // form in every tensor-core mode: a bias of that size in dW reaches nothing else.
    int spk_ = -1;                    // index into lay_.noise of that conv, or -1
    int spk_rows_ = 0;                // har rows per clip in the packed buffer (a multiple of s)
    Act har_full_;                    // har with its zero rows (har_ views the frames inside it)
    float* spk_dw_ = nullptr;         // weight gradient in packed form [Co][s*ld][taps]
    bool strided_tc(const ConvP& c) const {   // the weight gradient
        return spk_ >= 0 && &c == &lay_.noise[spk_] && tc_ok(c.s * pitch(c.cin), c.cout, 1);
    }
    bool strided_tc_fwd(const ConvP& c) const { return strided_tc(c) && tc_mode() != TC_TF32X3; }
    Act packed_view(const ConvP& c) const {
        Act a = har_full_;
        a.ld = c.s * har_full_.ld;
        a.C = a.ld;
        a.L = spk_rows_ / c.s;
        return a;
    }
    TcPlanes tc_planes(const Act& x, cudaStream_t st, int mode = -1);   // x -> planes in tc_xh_ / tc_xl_
    void tc_launch(const Act& x, const TcPlanes& xp, const float* whi, const float* wlo, int taps, int M,
                   const Act& y, const float* bias, const Act* r, int r_shift, int p, int d, int No, int o_base,
                   int orow_mul, int orow_off, float alpha, bool accum, double* stats, cudaStream_t st,
                   int mode = -1);
    PackJob* pack_jobs_ = nullptr;                // device: forward jobs, then dgrad jobs at PACK_MAX_JOBS
    int n_pack_fw_ = 0, n_pack_dg_ = 0, pack_jobs_math_ = -1;
    int64_t tot_pack_fw_ = 0, tot_pack_dg_ = 0;
    FcRow* fc_tab_ = nullptr;                     // device
    int* fc_row_entry_ = nullptr;                 // device
    int fc_rows_ = 0;
    int fc_tab_B_ = -1;

    // workspace (depends on B, T, frames)
    char* ws_ = nullptr;
    int64_t ws_bytes_ = 0;
    int B_ = 0, T_ = 0, frames_ = 0;
    bool have_har_ = false;
    bool planned_ = false;
    int plan_part_ = PART_FULL;       // what the plan covers
    bool plan_wg_ = false;            // the plan holds the weight gradients' plane copies (wg_split)
    int fwd_part_ = PART_FULL;        // what the last forward ran

    // per-call pointers
    const float* params_ = nullptr;
    float* grads_ = nullptr;
    const float* F0_ = nullptr;
    const float* N_ = nullptr;
    const float* style_ = nullptr;
    bool ref_mode_ = false;
    bool fwd_done_ = false;

    // planned buffers
    Act asr_, F0dn_, Ndn_, asrres_, enc_in_, har_, xl_, post_, genin_;
    std::vector<Act> dec_in_;
    BlkC encc_;
    RB1C rb1c_;                       // block mode: the AdaINResBlock1's caches
    Act blk_x_, blk_y_;               // block mode: channels-last input and output
    std::vector<BlkC> decc_;
    std::vector<char> res_applied_;
    std::vector<int> x_ch_;
    std::vector<StageC> stc_;
    float* aff_ = nullptr;
    float* daff_ = nullptr;
    float* spec_ = nullptr;
    float* hs_src_ = nullptr;
    double* hs_phase_ = nullptr;
    double* dacc_ = nullptr;          // reduction scratch (B * max C * 3)
    double* ssum_ = nullptr;          // per-(b, c) output sums of the last conv (B * max C * 2)
    double* bsum_ = nullptr;          // bias-gradient column sums (max C)
    double* bsum0_ = nullptr;         // column sums of a generator stage's resblock entry gradient
    float* part_ = nullptr;           // split-K partials
    int64_t part_floats_ = 0;
    float* fc_part_ = nullptr;
    Act S_[6];                        // backward scratch at the largest shape
    Act dasr_cl_, dasrres_, dF0dn_, dNdn_;
    float* F0_copy_ = nullptr;        // the forward's inputs, kept for the backward
    float* N_copy_ = nullptr;
    float* style_copy_ = nullptr;
};

}  // namespace bsml
