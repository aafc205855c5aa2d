// Decoder engine: the reference's decoder_backbone_forward_train / _backward and
// generator_forward_train / _backward (src/kokoro_decoder_backward.cpp:482-737),
// batched over clips, on channels-last device buffers, with the weight, bias,
// Snake-alpha, fc and input gradients the reference drops.
#include "engine.h"

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cmath>
#include <cstring>


namespace bsml {

namespace {

Act view(const Act& buf, int L, int C) {
    Act a = buf;
    a.L = L;
    a.C = C;
    a.ld = pitch(C);
    a.bstride = (int64_t)L * a.ld;
    return a;
}

// rows [r0, r0 + n) of an activation
Act rows(const Act& a, int r0, int n) {
    Act v = a;
    v.p = a.p + (int64_t)r0 * a.ld;
    v.L = n;
    return v;
}

Act flat_input(const float* p, int B, int L) {   // (B, L) as channels-last with C = 1, ld = 1
    Act a;
    a.p = const_cast<float*>(p);
    a.B = B; a.L = L; a.C = 1; a.ld = 1;
    a.bstride = L;
    return a;
}

int conv_out(int L, const ConvP& c) {
    const int64_t num = (int64_t)L + 2 * (int64_t)c.p - (int64_t)c.d * (c.k - 1) - 1;
    return num < 0 ? 0 : (int)(num / c.s + 1);
}

}  // namespace

namespace {
// NVTX range for the lifetime of the object: the engine's phases and conv calls
// show up by name in a profiler timeline (header-only NVTX; no cost without a tool)
struct Range {
    explicit Range(const char* n) { nvtxRangePushA(n); }
    ~Range() { nvtxRangePop(); }
    Range(const Range&) = delete;
    Range& operator=(const Range&) = delete;
};
}  // namespace

Engine::Engine(const bsml_decoder_config& cfg, int device) : lay_(cfg), device_(device) { init(); }
Engine::Engine(const bsml_block_spec& spec, int device) : lay_(spec), device_(device) { init(); }

void Engine::init() {
    BSML_CUDA(cudaSetDevice(device_));
    // packed weights: forward + dgrad layouts for every conv, phases + dgrad for every convT
    int64_t bytes = 0;
    auto sz = [&](int64_t floats) { bytes = round_up(bytes, 256) + floats * 4; };
    for (auto* c : lay_.convs) {
        sz((int64_t)c->k * c->cin * round_up(c->cout, 4));
        sz((int64_t)c->k * c->cout * round_up(c->cin, 4));
    }
    for (auto& u : lay_.ups) {
        for (int r = 0; r < u.s; ++r) sz((int64_t)((u.k - r + u.s - 1) / u.s) * u.cin * round_up(u.cout, 4));
        sz((int64_t)u.k * u.cout * round_up(u.cin, 4));
    }
    wp_bytes_ = round_up(bytes, 256);
    BSML_CUDA(cudaMalloc(&wp_mem_, wp_bytes_));
    int64_t off = 0;
    auto take = [&](int64_t floats) {
        off = round_up(off, 256);
        float* p = (float*)(wp_mem_ + off);
        off += floats * 4;
        return p;
    };
    wp_fwd_.resize(lay_.convs.size());
    wp_dgrad_.resize(lay_.convs.size());
    for (auto* c : lay_.convs) {
        wp_fwd_[c->id] = take((int64_t)c->k * c->cin * round_up(c->cout, 4));
        wp_dgrad_[c->id] = take((int64_t)c->k * c->cout * round_up(c->cin, 4));
    }
    wp_up_.resize(lay_.ups.size());
    wp_up_dgrad_.resize(lay_.ups.size());
    for (auto& u : lay_.ups) {
        for (int r = 0; r < u.s; ++r) wp_up_[u.id].push_back(take((int64_t)((u.k - r + u.s - 1) / u.s) * u.cin * round_up(u.cout, 4)));
        wp_up_dgrad_[u.id] = take((int64_t)u.k * u.cout * round_up(u.cin, 4));
    }
    // the first strided noise conv runs in row-packed form on the tensor cores
    for (size_t i = 0; i < lay_.noise.size(); ++i)
        if (lay_.noise[i].s > 1) {
            spk_ = (int)i;
            break;
        }
    // forward tensor-core planes of a conv: [k][Co][Ci] or, for the row-packed one, [ceil(k/s)][Co][s*ld]
    auto fwd_floats = [&](const ConvP* c) {
        int64_t n = (int64_t)c->k * c->cout * round_up(c->cin, 8);
        if (spk_ >= 0 && c == &lay_.noise[spk_])
            n = std::max<int64_t>(n, (int64_t)ceil_div(c->k, c->s) * c->cout * round_up((int64_t)c->s * pitch(c->cin), 8));
        return n;
    };
    // tensor-core weight planes: 2 fp32 planes per layout (bf16 uses the first half)
    {
        int64_t tb = 0;
        auto tsz = [&](int64_t floats) { tb = round_up(tb, 256) + floats * 4; };
        for (auto* c : lay_.convs) {
            tsz(fwd_floats(c)); tsz(fwd_floats(c));
            tsz((int64_t)c->k * c->cin * round_up(c->cout, 8)); tsz((int64_t)c->k * c->cin * round_up(c->cout, 8));
        }
        for (auto& u : lay_.ups) {
            for (int r = 0; r < u.s; ++r)
                for (int h = 0; h < 2; ++h) tsz((int64_t)((u.k - r + u.s - 1) / u.s) * u.cout * round_up(u.cin, 8));
            for (int h = 0; h < 2; ++h)
                tsz((int64_t)convT_pack(u.k, u.s, u.p).taps * u.cin * round_up((int64_t)u.s * u.cout, 8));
        }
        tcw_bytes_ = round_up(tb, 256);
        BSML_CUDA(cudaMalloc(&tcw_mem_, tcw_bytes_));
        int64_t toff = 0;
        auto ttake = [&](int64_t floats) {
            toff = round_up(toff, 256);
            float* p = (float*)(tcw_mem_ + toff);
            toff += floats * 4;
            return p;
        };
        const size_t nc = lay_.convs.size();
        tcw_fwd_hi_.resize(nc); tcw_fwd_lo_.resize(nc); tcw_dg_hi_.resize(nc); tcw_dg_lo_.resize(nc);
        for (auto* c : lay_.convs) {
            tcw_fwd_hi_[c->id] = ttake(fwd_floats(c));
            tcw_fwd_lo_[c->id] = ttake(fwd_floats(c));
            tcw_dg_hi_[c->id] = ttake((int64_t)c->k * c->cin * round_up(c->cout, 8));
            tcw_dg_lo_[c->id] = ttake((int64_t)c->k * c->cin * round_up(c->cout, 8));
        }
        tcw_up_hi_.resize(lay_.ups.size());
        tcw_up_lo_.resize(lay_.ups.size());
        tcw_updg_hi_.resize(lay_.ups.size());
        tcw_updg_lo_.resize(lay_.ups.size());
        for (auto& u : lay_.ups) {
            for (int r = 0; r < u.s; ++r) {
                const int64_t n = (int64_t)((u.k - r + u.s - 1) / u.s) * u.cout * round_up(u.cin, 8);
                tcw_up_hi_[u.id].push_back(ttake(n));
                tcw_up_lo_[u.id].push_back(ttake(n));
            }
            const int64_t n = (int64_t)convT_pack(u.k, u.s, u.p).taps * u.cin * round_up((int64_t)u.s * u.cout, 8);
            tcw_updg_hi_[u.id] = ttake(n);
            tcw_updg_lo_[u.id] = ttake(n);
        }
    }
    // fc row table (out offsets depend on B: rebuilt in ensure_plan)
    fc_rows_ = 0;
    for (int c : lay_.aff_C) fc_rows_ += 2 * c;
    BSML_CUDA(cudaMalloc(&fc_tab_, sizeof(FcRow) * lay_.aff_C.size()));
    BSML_CUDA(cudaMalloc(&fc_row_entry_, sizeof(int) * fc_rows_));
    std::vector<int> re(fc_rows_);
    int q = 0;
    for (size_t a = 0; a < lay_.aff_C.size(); ++a)
        for (int o = 0; o < 2 * lay_.aff_C[a]; ++o) re[q++] = (int)a;
    BSML_CUDA(cudaMemcpy(fc_row_entry_, re.data(), sizeof(int) * fc_rows_, cudaMemcpyHostToDevice));
    // the harmonic source depends only on F0: it runs on a second stream beside the backbone
    BSML_CUDA(cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking));
    BSML_CUDA(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
    BSML_CUDA(cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming));
}

Engine::~Engine() {
    cudaSetDevice(device_);
    for (auto ev : ev_pool_) cudaEventDestroy(ev);
    if (ev_fork_) cudaEventDestroy(ev_fork_);
    if (ev_join_) cudaEventDestroy(ev_join_);
    if (side_) cudaStreamDestroy(side_);
    cudaFree(wp_mem_);
    cudaFree(tcw_mem_);
    cudaFree(ws_);
    cudaFree(fc_tab_);
    cudaFree(fc_row_entry_);
    cudaFree(pack_jobs_);
}

void Engine::set_math(int m) {
    if (m != BSML_MATH_FP32_SIMT && m != BSML_MATH_TF32X3 && m != BSML_MATH_BF16 && m != BSML_MATH_BF16X3 &&
        m != BSML_MATH_TF32X3W && m != BSML_MATH_TF32X3F)
        fail("bsml_decoder_set_math", "unknown math mode " + std::to_string(m));
    math_ = m;
}

void Engine::set_profiling(bool on) { prof_on_ = on; }

void Engine::set_phase_mode(int m) {
    if (m != PHASE_FP32_RUNNING && m != PHASE_EXACT)
        fail("bsml_decoder_set_phase_mode", "unknown phase mode " + std::to_string(m));
    phase_mode_ = m;
}

int Engine::prof_begin(int cls, double work, cudaStream_t st) {
    if (!prof_on_) return -1;
    while (ev_pool_.size() < ev_used_ + 2) {
        cudaEvent_t e;
        BSML_CUDA(cudaEventCreate(&e));
        ev_pool_.push_back(e);
    }
    ProfRec r{cls, work, ev_pool_[ev_used_], ev_pool_[ev_used_ + 1]};
    ev_used_ += 2;
    BSML_CUDA(cudaEventRecord(r.a, st));
    prof_.push_back(r);
    return (int)prof_.size() - 1;
}

void Engine::prof_end(int id, cudaStream_t st) {
    if (id >= 0) BSML_CUDA(cudaEventRecord(prof_[id].b, st));
}

void Engine::read_profile_records(double* out, int max_records, int* n_records) {
    BSML_CUDA(cudaDeviceSynchronize());
    int n = 0;
    for (auto& r : prof_) {
        if (n >= max_records) break;
        float ms = 0;
        BSML_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        out[3 * n] = r.cls;
        out[3 * n + 1] = r.work;
        out[3 * n + 2] = ms;
        ++n;
    }
    *n_records = n;
    prof_.clear();
    ev_used_ = 0;
}

void Engine::read_profile(double* out) {
    for (int i = 0; i < PROF_N * 3; ++i) out[i] = 0;
    BSML_CUDA(cudaDeviceSynchronize());
    for (auto& r : prof_) {
        float ms = 0;
        BSML_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        out[r.cls * 3] += ms;
        out[r.cls * 3 + 1] += r.work;
        out[r.cls * 3 + 2] += 1;
    }
    prof_.clear();
    ev_used_ = 0;
}

Engine::Stats Engine::stats(Planner& P, int B, int C) {
    Stats s;
    s.mean = P.f((int64_t)B * C);
    s.rstd = P.f((int64_t)B * C);
    return s;
}

Engine::BlkC Engine::plan_blk(Planner& P, const BlkP& w, int Lin, bool) {
    BlkC c;
    c.Lin = Lin;
    c.Lout = w.up ? 2 * Lin : Lin;
    c.s1 = stats(P, B_, w.cin);
    c.s2 = stats(P, B_, w.cout);
    c.r = P.act(B_, Lin, w.cin);
    if (w.up) c.pooled = P.act(B_, c.Lout, w.cin);
    c.c1 = P.act(B_, c.Lout, w.cout);
    c.n2 = P.act(B_, c.Lout, w.cout);
    if (w.sc) c.sc = P.act(B_, Lin, w.cout);
    return c;
}

Engine::RB1C Engine::plan_rb1(Planner& P, int L, int C) {
    RB1C c;
    c.L = L;
    for (int i = 0; i < 3; ++i) {
        if (i > 0) c.x[i] = P.act(B_, L, C);
        c.c1[i] = P.act(B_, L, C);
        c.st1[i] = stats(P, B_, C);
        c.st2[i] = stats(P, B_, C);
    }
    return c;
}

void Engine::plan(Planner& P) {
    const auto& cf = lay_.cfg;
    const int B = B_, T = T_;
    int64_t max_elems = 0;
    int max_c = 0;
    auto note = [&](int L, int C) {
        max_elems = std::max<int64_t>(max_elems, (int64_t)B * L * pitch(C));
        max_c = std::max(max_c, C);
    };
    style_copy_ = P.f((int64_t)B * cf.style_dim);
    aff_ = P.f((int64_t)B * lay_.aff_per_clip);
    daff_ = P.f((int64_t)B * lay_.aff_per_clip);
    int L = T;
    if (plan_part_ != PART_GENERATOR) {
        asr_ = P.act(B, T, cf.asr_dim);
        F0_copy_ = P.f((int64_t)B * 2 * T);
        N_copy_ = P.f((int64_t)B * 2 * T);
        F0dn_ = P.act(B, T, 1);
        Ndn_ = P.act(B, T, 1);
        asrres_ = P.act(B, T, cf.asr_res_dim);
        enc_in_ = P.act(B, T, cf.asr_dim + 2);
        encc_ = plan_blk(P, lay_.enc, T, true);
        encc_.x = enc_in_;
        note(T, lay_.enc.cin);
        note(T, lay_.enc.cout);
        const int nd = (int)lay_.dec.size();
        dec_in_.resize(nd);
        decc_.resize(nd);
        res_applied_.assign(nd, 0);
        x_ch_.assign(nd, 0);
        int Cx = cf.enc_dim;
        bool res = true;
        for (int i = 0; i < nd; ++i) {
            const BlkP& w = lay_.dec[i];
            x_ch_[i] = Cx;
            res_applied_[i] = res ? 1 : 0;
            dec_in_[i] = P.act(B, L, w.cin);
            decc_[i] = plan_blk(P, w, L, true);
            decc_[i].x = dec_in_[i];
            note(L, w.cin);
            note(decc_[i].Lout, w.cin);
            note(decc_[i].Lout, w.cout);
            L = decc_[i].Lout;
            Cx = w.cout;
            if (w.up) res = false;
        }
        // backward-only buffers
        dasr_cl_ = P.act(B, T, cf.asr_dim);
        dasrres_ = P.act(B, T, cf.asr_res_dim);
        dF0dn_ = P.act(B, T, 1);
        dNdn_ = P.act(B, T, 1);
    }
    // the generator part on its own takes gen_in of length T_ (its L_in)
    genin_ = P.act(B, L, cf.init_ch);
    note(L, cf.init_ch);
    if (plan_part_ == PART_BACKBONE) {
        plan_scratch(P, max_elems, max_c);
        return;
    }
    // harmonic source / har
    const int Fr = 2 * T;
    if (!have_har_) {
        frames_ = (Fr * cf.upsample_scale) / cf.hop + 1;
        hs_phase_ = P.d((int64_t)B * (cf.harmonic_num + 1) * Fr);
        hs_src_ = P.f((int64_t)B * Fr * cf.upsample_scale);
    }
    if (spk_ >= 0) {
        // rows [0, p) and [p + frames, R) stay zero; the packed conv reads rows < s * (No + taps - 1)
        const ConvP& c = lay_.noise[spk_];
        const int No = conv_out(frames_, c);
        const int64_t need = std::max<int64_t>((int64_t)c.s * (No + ceil_div(c.k, c.s) - 1), (int64_t)c.p + frames_);
        spk_rows_ = (int)round_up(need, c.s);
        har_full_ = P.act(B, spk_rows_, cf.har_ch);
        har_ = har_full_;
        har_.p = har_full_.p ? har_full_.p + (int64_t)c.p * har_full_.ld : nullptr;
        har_.L = frames_;
        note(spk_rows_, cf.har_ch);
        spk_dw_ = P.f((int64_t)c.cout * c.s * pitch(c.cin) * ceil_div(c.k, c.s));
    } else {
        har_ = P.act(B, frames_, cf.har_ch);
    }
    // generator stages
    const int U = cf.n_ups, K = cf.n_kernels;
    stc_.assign(U, StageC{});
    for (int i = 0; i < U; ++i) {
        StageC& s = stc_[i];
        const UpP& u = lay_.ups[i];
        s.Lin = L;
        s.x_in = (i == 0) ? genin_ : stc_[i - 1].out;
        s.a = P.act(B, L, u.cin);
        s.Lu = (L - 1) * u.s - 2 * u.p + u.k;
        s.Lx = s.Lu + (i == U - 1 ? 1 : 0);
        const int Lsrc = conv_out(frames_, lay_.noise[i]);
        if (Lsrc != s.Lx)
            fail("bsml_decoder_forward", "noise source length " + std::to_string(Lsrc) + " != upsampled length " +
                                             std::to_string(s.Lx) + " at stage " + std::to_string(i));
        s.xsrc = P.act(B, s.Lx, u.cout);
        s.src = P.act(B, s.Lx, u.cout);
        s.m = P.act(B, s.Lx, u.cout);
        s.out = P.act(B, s.Lx, u.cout);
        s.noise = plan_rb1(P, s.Lx, u.cout);
        s.noise.x[0] = s.xsrc;
        s.res.resize(K);
        for (int j = 0; j < K; ++j) {
            s.res[j] = plan_rb1(P, s.Lx, u.cout);
            s.res[j].x[0] = s.m;
            if (j > 0) s.res[j].st1[0] = s.res[0].st1[0];   // same input, same statistics
        }
        note(L, u.cin);
        note(s.Lx, u.cout);
        L = s.Lx;
    }
    xl_ = P.act(B, L, lay_.post.cin);
    post_ = P.act(B, L, lay_.post.cout);
    spec_ = P.f((int64_t)B * L * (cf.n_fft + 2));
    note(L, lay_.post.cout);
    plan_scratch(P, max_elems, max_c);
}

// reduction scratch, split-K partials, the backward's scratch activations and
// the tensor-core operand planes, sized for the largest activation
void Engine::plan_scratch(Planner& P, int64_t max_elems, int max_c) {
    const int B = B_;
    const auto& cf = lay_.cfg;
    dacc_ = P.d((int64_t)B * std::max(max_c, 1) * 3);
    ssum_ = P.d((int64_t)B * std::max(max_c, 1) * 2);
    bsum_ = P.d(std::max(max_c, 1));
    bsum0_ = P.d(std::max(max_c, 1));
    part_floats_ = 48ll << 20;
    part_ = P.f(part_floats_);
    fc_part_ = P.f(ceil_div(fc_rows_, 256) * (int64_t)B * cf.style_dim + 64);
    for (Act& s : S_) {
        s = Act{};
        s.B = B;
        s.p = P.f(max_elems);
    }
    // activation operand planes for the tensor-core path (largest conv input)
    tc_xh_ = P.f(max_elems);
    tc_xl_ = P.f(max_elems);
    tc_yh_ = P.f(max_elems);
    tc_yl_ = P.f(max_elems);
    tc_dh_ = P.f(max_elems);
    tc_dl_ = P.f(max_elems);
    tc_eh_ = P.f(max_elems);
    tc_el_ = P.f(max_elems);
    // the weight gradients' copies (bf16 hi + lo, 4 bytes per element: fits max_elems
    // floats per plane even with the bf16 pitch's rounding to 8 channels)
    const int64_t wn = plan_wg_ ? max_elems : 64;
    tc_dwh_ = P.f(wn);
    tc_dwl_ = P.f(wn);
    tc_uwh_ = P.f(wn);
    tc_uwl_ = P.f(wn);
    tc_ewh_ = P.f(wn);
    tc_ewl_ = P.f(wn);
}

// One block (block_kind != 0): T_ is the block's input length L
void Engine::plan_block(Planner& P) {
    const int B = B_, L = T_;
    style_copy_ = P.f((int64_t)B * lay_.cfg.style_dim);
    aff_ = P.f((int64_t)B * lay_.aff_per_clip);
    daff_ = P.f((int64_t)B * lay_.aff_per_clip);
    int64_t max_elems = 0;
    int max_c = 0;
    if (lay_.block_kind == BSML_BLOCK_RESBLK1D) {
        const BlkP& w = lay_.enc;
        blk_x_ = P.act(B, L, w.cin);
        encc_ = plan_blk(P, w, L, true);
        encc_.x = blk_x_;
        blk_y_ = P.act(B, encc_.Lout, w.cout);
        max_c = std::max(w.cin, w.cout);
        max_elems = (int64_t)B * encc_.Lout * pitch(max_c);
    } else {
        const RB1P& w = lay_.rbs[0];
        blk_x_ = P.act(B, L, w.C);
        rb1c_ = plan_rb1(P, L, w.C);
        rb1c_.x[0] = blk_x_;
        blk_y_ = P.act(B, L, w.C);
        max_c = w.C;
        max_elems = (int64_t)B * L * pitch(w.C);
    }
    plan_scratch(P, max_elems, max_c);
}

void Engine::ensure_plan(int B, int T, int frames, bool have_har, int part) {
    if (planned_ && B == B_ && T == T_ && part == plan_part_ && have_har == have_har_ &&
        (!have_har || frames == frames_) && plan_wg_ == wg_split())
        return;
    B_ = B; T_ = T; frames_ = frames; have_har_ = have_har; plan_part_ = part; plan_wg_ = wg_split();
    Planner p0;
    if (lay_.block_kind) plan_block(p0);
    else plan(p0);
    const int64_t need = round_up(p0.off, 1 << 20);
    if (need > ws_bytes_) {
        if (ws_) BSML_CUDA(cudaFree(ws_));
        ws_ = nullptr;
        ws_bytes_ = 0;
        BSML_CUDA(cudaMalloc(&ws_, need));
        ws_bytes_ = need;
    }
    Planner p1;
    p1.base = ws_;
    if (lay_.block_kind) plan_block(p1);
    else plan(p1);
    // fc table for this B
    std::vector<FcRow> tab(lay_.aff_C.size());
    int row0 = 0;
    auto fill_tab = [&](const AdaP& a) {
        FcRow& f = tab[a.idx];
        f.w_off = a.fw;
        f.b_off = a.fb;
        f.out_off = (int64_t)B * lay_.aff_base[a.idx];
        f.n_out = 2 * a.C;
    };
    for (const AdaP* a : lay_.adains) fill_tab(*a);
    for (auto& f : tab) { f.row0 = row0; row0 += f.n_out; }
    BSML_CUDA(cudaMemcpy(fc_tab_, tab.data(), sizeof(FcRow) * tab.size(), cudaMemcpyHostToDevice));
    planned_ = true;
}

// ── weight packing (every step: the parameters may have changed). The tensor-core
// packings of one direction run as one batched launch; the job tables depend only
// on the math mode and are built on first use.
void Engine::build_pack_jobs() {
    std::vector<PackJob> fw, dg;
    auto add = [](std::vector<PackJob>& v, const PackJob& J) {
        PackJob j = J;
        j.start = v.empty() ? 0 : v.back().start + v.back().items;
        v.push_back(j);
    };
    if (math_ != BSML_MATH_FP32_SIMT) {
        for (auto* c : lay_.convs) {
            if (tc_ok(c->cin, c->cout, c->s))
                add(fw, make_pack_job(c->w, PACK_CONV_FWD, c->cout, c->cin, c->k, 1, 0, tcw_fwd_hi_[c->id],
                                      tcw_fwd_lo_[c->id]));
            else if (strided_tc_fwd(*c))
                add(fw, make_pack_job(c->w, PACK_CONV_STRIDED, c->cout, c->cin, c->k, c->s, pitch(c->cin),
                                      tcw_fwd_hi_[c->id], tcw_fwd_lo_[c->id]));
            if (c->s == 1 && tc_ok(c->cout, c->cin, 1))
                add(dg, make_pack_job(c->w, PACK_CONV_DGRAD, c->cout, c->cin, c->k, 1, 0, tcw_dg_hi_[c->id],
                                      tcw_dg_lo_[c->id]));
        }
        for (auto& u : lay_.ups) {
            if (tc_ok(u.cin, u.cout, 1))
                for (int r = 0; r < u.s; ++r)
                    add(fw, make_pack_job(u.w, PACK_CONVT_PHASE, u.cout, u.cin, u.k, u.s, r, tcw_up_hi_[u.id][r],
                                          tcw_up_lo_[u.id][r]));
            if (convT_tc(u))
                add(dg, make_pack_job(u.w, PACK_CONVT_DGRAD, u.cout, u.cin, u.k, u.s, u.p, tcw_updg_hi_[u.id],
                                      tcw_updg_lo_[u.id]));
        }
    }
    if (fw.size() > (size_t)PACK_MAX_JOBS || dg.size() > (size_t)PACK_MAX_JOBS)
        fail("bsml_decoder", "too many tensor-core weight packings for one batch");
    if (!pack_jobs_) BSML_CUDA(cudaMalloc(&pack_jobs_, sizeof(PackJob) * 2 * PACK_MAX_JOBS));
    if (!fw.empty()) BSML_CUDA(cudaMemcpy(pack_jobs_, fw.data(), sizeof(PackJob) * fw.size(), cudaMemcpyHostToDevice));
    if (!dg.empty())
        BSML_CUDA(cudaMemcpy(pack_jobs_ + PACK_MAX_JOBS, dg.data(), sizeof(PackJob) * dg.size(),
                             cudaMemcpyHostToDevice));
    n_pack_fw_ = (int)fw.size();
    n_pack_dg_ = (int)dg.size();
    tot_pack_fw_ = fw.empty() ? 0 : fw.back().start + fw.back().items;
    tot_pack_dg_ = dg.empty() ? 0 : dg.back().start + dg.back().items;
    pack_jobs_math_ = math_;
}

void Engine::pack_weights(cudaStream_t st) {
    if (pack_jobs_math_ != math_) build_pack_jobs();
    pack_w_tc_batch(params_, pack_jobs_, n_pack_fw_, tot_pack_fw_, tc_mode(), st);
    for (auto* c : lay_.convs)
        if (!tc_ok(c->cin, c->cout, c->s) && !strided_tc_fwd(*c))
            pack_conv_fwd(params_ + c->w, c->cout, c->cin, c->k, wp_fwd_[c->id], st);
    for (auto& u : lay_.ups)
        if (!tc_ok(u.cin, u.cout, 1))
            for (int r = 0; r < u.s; ++r) pack_convT_phase(params_ + u.w, u.cin, u.cout, u.k, u.s, r, wp_up_[u.id][r], st);
}
void Engine::pack_dgrad_weights(cudaStream_t st) {
    if (pack_jobs_math_ != math_) build_pack_jobs();
    pack_w_tc_batch(params_, pack_jobs_ + PACK_MAX_JOBS, n_pack_dg_, tot_pack_dg_, bw_mode(), st);
    for (auto* c : lay_.convs)
        if (c->s == 1 && !tc_ok(c->cout, c->cin, 1))
            pack_conv_dgrad(params_ + c->w, c->cout, c->cin, c->k, wp_dgrad_[c->id], st);
    // the CUDA-core convT input gradient is the fallback when L_u % s != 0
    for (auto& u : lay_.ups) pack_convT_dgrad(params_ + u.w, u.cin, u.cout, u.k, wp_up_dgrad_[u.id], st);
}

TcPlanes Engine::tc_planes(const Act& x, cudaStream_t st, int mode) {
    if (!x.p) fail("conv", "internal: operand has neither fp32 data nor planes");
    if (mode < 0) mode = tc_mode();
    make_act_planes(x, mode, tc_xh_, tc_xl_, st);
    TcPlanes t;
    t.hi = tc_xh_; t.lo = tc_xl_; t.ld = tc_pitch(x.C, mode);
    return t;
}

Engine::Opnd Engine::operand(bool tc, int L, int C, const Act& fbuf, void* hi, void* lo, int mode) const {
    Opnd o;
    o.f = view(fbuf, L, C);
    if (tc) {
        o.f.p = nullptr;
        o.tp.hi = hi; o.tp.lo = lo; o.tp.ld = tc_pitch(C, mode < 0 ? tc_mode() : mode);
    }
    return o;
}

void Engine::adain_fwd_to(const Act& x, const double* sums, const Stats& s, const float* gb, int act, float slope,
                          const float* alpha, const Opnd& out, cudaStream_t st) {
    PlaneOut po;
    po.hi = const_cast<void*>(out.tp.hi); po.lo = const_cast<void*>(out.tp.lo); po.ld = out.tp.ld; po.mode = tc_mode();
    adain_act_fwd_v(x, sums, 1e-5f, s.mean, s.rstd, gb, act, slope, alpha, out.f.p ? &out.f : nullptr,
                    out.tp.hi ? &po : nullptr, st);
}

void Engine::adain_bwd_to(const Act& x, const Stats& s, const float* gb, int act, float slope, const float* alpha,
                          const Act& dy, const Opnd& out, const Act* skip, double* colsum, float* dgb, float* dalpha,
                          cudaStream_t st, bool acc_ready, float skip_scale, bool out_accum) {
    PlaneOut po, po2;
    po.hi = const_cast<void*>(out.tp.hi); po.lo = const_cast<void*>(out.tp.lo); po.ld = out.tp.ld; po.mode = bw_mode();
    po2.hi = const_cast<void*>(out.tpw.hi); po2.lo = const_cast<void*>(out.tpw.lo); po2.ld = out.tpw.ld;
    po2.mode = wg_mode();
    adain_act_bwd_v(x, s.mean, s.rstd, gb, act, slope, alpha, dy, out.f.p ? &out.f : nullptr, skip,
                    out.tp.hi ? &po : nullptr, colsum, dgb, dalpha, dacc_, st, acc_ready, skip_scale, out_accum,
                    out.tpw.hi ? &po2 : nullptr);
}

void Engine::recompute_reduce_to(const Act& x, const Stats& s, const float* gb, int act, float slope,
                                 const float* alpha, const Act& dy, const Opnd& out, cudaStream_t st) {
    PlaneOut po;
    po.hi = const_cast<void*>(out.tp.hi); po.lo = const_cast<void*>(out.tp.lo); po.ld = out.tp.ld; po.mode = wg_mode();
    adain_recompute_reduce(x, s.mean, s.rstd, gb, act, slope, alpha, out.f.p ? &out.f : nullptr,
                           out.tp.hi ? &po : nullptr, dy, dacc_, st);
}

void Engine::tc_launch(const Act& x, const TcPlanes& xp, const float* whi, const float* wlo, int taps, int M,
                       const Act& y, const float* bias, const Act* r, int r_shift, int p, int d, int No, int o_base,
                       int orow_mul, int orow_off, float alpha, bool accum, double* stats, cudaStream_t st,
                       int mode) {
    TcConvFwd a;
    a.x = xp;
    a.B = x.B; a.L_in = x.L; a.Ci = x.C;
    a.w.hi = whi; a.w.lo = wlo; a.w.ld = (int)round_up(x.C, 8);
    a.taps = taps; a.Co = M;
    a.p = p; a.d = d; a.No = No; a.o_base = o_base;
    a.y = y; a.bias = bias; a.r = r; a.r_shift = r_shift; a.orow_mul = orow_mul; a.orow_off = orow_off;
    a.alpha = alpha; a.accum = accum;
    a.stats = stats;
    a.part = part_; a.part_cap = part_floats_;   // split-K scratch, shared with the weight gradients
    conv_fwd_tc(a, mode < 0 ? tc_mode() : mode, st);
}

// ── conv wrappers
void Engine::conv(const ConvP& c, const Act& x, const Act& y, const Act* r, int r_shift, float alpha, bool accum,
                  cudaStream_t st, const TcPlanes* xp, double* stats) {
    const Range nvtx_range("bsml.conv.fwd");
    ConvFwd a;
    a.x = x; a.y = y; a.wp = wp_fwd_[c.id]; a.bias = P(c.b); a.r = r; a.r_shift = r_shift;
    a.k = c.k; a.s = c.s; a.p = c.p; a.d = c.d;
    a.No = conv_out(x.L, c);
    a.alpha = alpha; a.accum = accum;
    if (a.No != y.L) fail("conv", "output length mismatch");
    if (stats) BSML_CUDA(cudaMemsetAsync(stats, 0, sizeof(double) * 2 * (size_t)y.B * c.cout, st));
    if (strided_tc_fwd(c)) {
        // x is har_, a view inside har_full_: the packed rows start at the buffer's first (zero) row
        const Act X2 = packed_view(c);
        const TcPlanes tp = tc_planes(X2, st);
        const int id = prof_begin(PROF_CONV_TC, 2.0 * c.cin * c.cout * c.k * (double)a.No * x.B, st);
        tc_launch(X2, tp, tcw_fwd_hi_[c.id], tcw_fwd_lo_[c.id], (int)ceil_div(c.k, c.s), c.cout, y, a.bias, r,
                  r_shift, 0, 1, a.No, 0, 1, 0, alpha, accum, stats, st);
        prof_end(id, st);
        return;
    }
    if (tc_ok(c.cin, c.cout, c.s)) {
        const TcPlanes tp = xp ? *xp : tc_planes(x, st);
        const int id = prof_begin(PROF_CONV_TC, 2.0 * c.cin * c.cout * c.k * (double)a.No * x.B, st);
        tc_launch(x, tp, tcw_fwd_hi_[c.id], tcw_fwd_lo_[c.id], c.k, c.cout, y, a.bias, r, r_shift, c.p, c.d, a.No, 0,
                  1, 0, alpha, accum, stats, st);
        prof_end(id, st);
        return;
    }
    if (!x.p) fail("conv", "internal: fp32 operand missing on the CUDA-core path");
    const int id = prof_begin(PROF_CONV_SIMT, 2.0 * c.cin * c.cout * c.k * (double)a.No * x.B, st);
    conv_fwd_simt(a, st);
    prof_end(id, st);
    if (stats) norm_sums(y, stats, st);
}

// dx[j] = sum_{t,co} W[co,ci,t] dy[j + p - t*d]: a forward conv over dy with the
// flipped, transposed weight and padding d*(k-1) - p (stride 1 only).
void Engine::conv_dgrad(const ConvP& c, const Act& dy, const Act& dx, bool accum, cudaStream_t st,
                        const TcPlanes* dyp) {
    const Range nvtx_range("bsml.conv.dgrad");
    if (c.s != 1) fail("conv_dgrad", "strided conv input gradients are not needed on this path");
    ConvFwd a;
    a.x = dy; a.y = dx; a.wp = wp_dgrad_[c.id];
    a.k = c.k; a.s = 1; a.p = c.d * (c.k - 1) - c.p; a.d = c.d;
    a.No = dx.L;
    a.accum = accum;
    if (tc_ok(c.cout, c.cin, 1)) {
        const TcPlanes tp = dyp ? *dyp : tc_planes(dy, st, bw_mode());
        const int id = prof_begin(PROF_CONV_TC, 2.0 * c.cin * c.cout * c.k * (double)dy.L * dy.B, st);
        tc_launch(dy, tp, tcw_dg_hi_[c.id], tcw_dg_lo_[c.id], c.k, c.cin, dx, nullptr, nullptr, 0, a.p, c.d, a.No, 0,
                  1, 0, 1.f, accum, nullptr, st, bw_mode());
        prof_end(id, st);
        return;
    }
    if (!dy.p) fail("conv_dgrad", "internal: fp32 operand missing on the CUDA-core path");
    const int id = prof_begin(PROF_CONV_SIMT, 2.0 * c.cin * c.cout * c.k * (double)dy.L * dy.B, st);
    conv_fwd_simt(a, st);
    prof_end(id, st);
}

void Engine::conv_wgrad(const ConvP& c, const Act& dy, const Act& x, cudaStream_t st, const TcPlanes* dyp,
                        const TcPlanes* xp, const double* bias_sum) {
    const Range nvtx_range("bsml.conv.wgrad");
    if (!grads_) return;
    // dyp / xp: planes in wg_mode(); otherwise they are made here from the fp32 data
    if (strided_tc(c)) {
        const int mode = wg_mode();
        const Act X2 = packed_view(c);
        TcConvWgrad w;
        if (dyp) {
            w.dy = *dyp;
        } else {
            make_act_planes(dy, mode, tc_yh_, tc_yl_, st);
            w.dy.hi = tc_yh_; w.dy.lo = tc_yl_; w.dy.ld = tc_pitch(dy.C, mode);
        }
        w.x = tc_planes(X2, st, mode);
        w.B = dy.B; w.Lo = dy.L; w.Co = dy.C; w.L_in = X2.L; w.Ci = X2.C;
        w.taps = (int)ceil_div(c.k, c.s); w.p = 0; w.d = 1; w.dW = spk_dw_;
        const int id = prof_begin(PROF_WGRAD_TC, 2.0 * c.cin * c.cout * c.k * (double)dy.L * dy.B, st);
        conv_wgrad_tc(w, mode, part_, part_floats_, st);
        wgrad_unpack_strided(spk_dw_, c.cout, c.cin, c.k, c.s, har_full_.ld, grads_ + c.w, st);
        if (c.b >= 0) {
            if (bias_sum) d2f(bias_sum, c.cout, grads_ + c.b, false, st);
            else colsum(dy, grads_ + c.b, false, part_, st);
        }
        prof_end(id, st);
        return;
    }
    if (tc_ok(c.cin, c.cout, c.s)) {
        const int mode = wg_mode();
        TcConvWgrad w;
        if (dyp) {
            w.dy = *dyp;
        } else {
            if (!dy.p) fail("conv_wgrad", "internal: operand has neither fp32 data nor planes");
            make_act_planes(dy, mode, tc_yh_, tc_yl_, st);
            w.dy.hi = tc_yh_; w.dy.lo = tc_yl_; w.dy.ld = tc_pitch(dy.C, mode);
        }
        w.x = xp ? *xp : tc_planes(x, st, mode);
        w.B = dy.B; w.Lo = dy.L; w.Co = dy.C; w.L_in = x.L; w.Ci = x.C;
        w.taps = c.k; w.p = c.p; w.d = c.d; w.dW = grads_ + c.w;
        const int id = prof_begin(PROF_WGRAD_TC, 2.0 * c.cin * c.cout * c.k * (double)dy.L * dy.B, st);
        conv_wgrad_tc(w, mode, part_, part_floats_, st);
        if (c.b >= 0) {
            if (bias_sum) d2f(bias_sum, c.cout, grads_ + c.b, false, st);
            else if (dy.p) colsum(dy, grads_ + c.b, false, part_, st);
            else fail("conv_wgrad", "internal: bias gradient needs fp32 dy or its column sums");
        }
        prof_end(id, st);
        return;
    }
    if (!dy.p || !x.p) fail("conv_wgrad", "internal: fp32 operand missing on the CUDA-core path");
    ConvWgrad a;
    a.dy = dy; a.x = x; a.k = c.k; a.s = c.s; a.p = c.p; a.d = c.d;
    a.dW = grads_ + c.w;
    a.db = bias_sum ? nullptr : G(c.b);
    if (wgrad_partial_floats(a) > part_floats_) fail("conv_wgrad", "split-K partial buffer too small");
    const int id = prof_begin(PROF_WGRAD_SIMT, 2.0 * c.cin * c.cout * c.k * (double)dy.L * dy.B, st);
    conv_wgrad_simt(a, part_, st);
    if (bias_sum && c.b >= 0) d2f(bias_sum, c.cout, grads_ + c.b, false, st);
    prof_end(id, st);
}

// ConvTranspose1d forward as one forward conv per stride phase r:
//   y[q*s + r - p] = sum_m sum_ci W[ci, co, r + m*s] x[q - m, ci]
void Engine::convT(const UpP& u, const Act& x, const Act& y, int row_off, const Act* r, cudaStream_t st) {
    const Range nvtx_range("bsml.convT.fwd");
    const int Lu = (x.L - 1) * u.s - 2 * u.p + u.k;
    const bool tc = tc_ok(u.cin, u.cout, 1);
    TcPlanes tp;
    if (tc) tp = tc_planes(x, st);
    for (int ph = 0; ph < u.s; ++ph) {
        const int kr = (u.k - ph + u.s - 1) / u.s;
        if (kr <= 0) continue;
        // q with 0 <= q*s + ph - p < Lu
        const int qmin = (int)ceil_div(std::max(u.p - ph, 0), u.s);
        const int qmax = (Lu - 1 + u.p - ph) >= 0 ? (Lu - 1 + u.p - ph) / u.s : -1;
        if (qmax < qmin) continue;
        ConvFwd a;
        a.x = x; a.y = y; a.wp = wp_up_[u.id][ph]; a.bias = P(u.b); a.r = r;
        a.k = kr; a.s = 1; a.p = kr - 1; a.d = 1;
        a.No = qmax - qmin + 1; a.o_base = qmin;
        a.orow_mul = u.s; a.orow_off = ph - u.p + row_off;
        const int id = prof_begin(tc ? PROF_CONV_TC : PROF_CONV_SIMT, 2.0 * u.cin * u.cout * kr * (double)a.No * x.B, st);
        if (tc)
            tc_launch(x, tp, tcw_up_hi_[u.id][ph], tcw_up_lo_[u.id][ph], kr, u.cout, y, a.bias, r, 0, a.p, 1, a.No,
                      a.o_base, a.orow_mul, a.orow_off, 1.f, false, nullptr, st);
        else
            conv_fwd_simt(a, st);
        prof_end(id, st);
    }
}

// dx[l, ci] = sum_{t, co} W[ci, co, t] dy[l*s - p + t, co]. Tensor cores: a stride-1
// conv over dy viewed row-packed (ConvTPack: K = s*Co, taps u_min..u_max); CUDA
// cores: a strided forward conv over dy.
void Engine::convT_dgrad(const UpP& u, const Act& dy, const Act& dx, cudaStream_t st, const TcPlanes* dyp) {
    const Range nvtx_range("bsml.convT.dgrad");
    if (dyp) {
        const ConvTPack pk = convT_pack(u.k, u.s, u.p);
        TcConvFwd a;
        a.x.hi = dyp->hi; a.x.lo = dyp->lo; a.x.ld = u.s * u.cout;
        a.B = dy.B; a.L_in = dy.L / u.s; a.Ci = u.s * u.cout;
        a.w.hi = tcw_updg_hi_[u.id]; a.w.lo = tcw_updg_lo_[u.id]; a.w.ld = (int)round_up((int64_t)u.s * u.cout, 8);
        a.taps = pk.taps; a.Co = u.cin;
        a.p = -pk.u_min; a.d = 1; a.No = dx.L; a.o_base = 0;
        a.y = dx;
        a.part = part_; a.part_cap = part_floats_;
        const int id = prof_begin(PROF_CONV_TC, 2.0 * u.cin * u.cout * u.k * (double)dx.L * dx.B, st);
        conv_fwd_tc(a, bw_mode(), st);
        prof_end(id, st);
        return;
    }
    ConvFwd a;
    a.x = dy; a.y = dx; a.wp = wp_up_dgrad_[u.id];
    a.k = u.k; a.s = u.s; a.p = u.p; a.d = 1;
    a.No = dx.L;
    const int id = prof_begin(PROF_CONV_SIMT, 2.0 * u.cin * u.cout * u.k * (double)dx.L * dx.B, st);
    conv_fwd_simt(a, st);
    prof_end(id, st);
}

// dW[ci, co, t] = sum x[l, ci] dy[l*s - p + t, co] (conv wgrad with roles swapped; on
// the tensor cores over the row-packed dy), db = colsum(dy)
void Engine::convT_wgrad(const UpP& u, const Act& dy, const Act& x, cudaStream_t st, const TcPlanes* dyp) {
    const Range nvtx_range("bsml.convT.wgrad");
    if (!grads_) return;
    if (dyp) {
        // dyp: the input gradient's row-packed planes (tc_mode); under wg_split the
        // weight gradient's are made again from dy in wg_mode (same buffers: the input
        // gradient has already read them)
        const ConvTPack pk = convT_pack(u.k, u.s, u.p);
        const int mode = wg_mode();
        TcConvWgrad w;
        w.dy = tc_planes(x, st, mode);   // the convT input plays dY's role (M = Ci of the convT)
        if (wg_split()) {
            if (tc_pitch(dy.C, mode) != dy.C) fail("convT_wgrad", "internal: row-packed planes need compact rows");
            make_act_planes(dy, mode, tc_yh_, tc_yl_, st);
            w.x.hi = tc_yh_; w.x.lo = tc_yl_;
        } else {
            w.x = *dyp;
        }
        w.x.ld = u.s * u.cout;
        w.B = x.B; w.Lo = x.L; w.Co = u.cin; w.L_in = dy.L / u.s; w.Ci = u.s * u.cout;
        w.taps = pk.taps; w.p = -pk.u_min; w.d = 1;
        w.dW = grads_ + u.w;
        w.ct_s = u.s; w.ct_p = u.p; w.ct_k = u.k; w.ct_Co = u.cout;
        const int id = prof_begin(PROF_WGRAD_TC, 2.0 * u.cin * u.cout * u.k * (double)x.L * x.B, st);
        conv_wgrad_tc(w, mode, part_, part_floats_, st);
        colsum(dy, grads_ + u.b, false, part_, st);
        prof_end(id, st);
        return;
    }
    ConvWgrad a;
    a.dy = x; a.x = dy; a.k = u.k; a.s = u.s; a.p = u.p; a.d = 1;
    a.dW = grads_ + u.w;
    a.db = nullptr;
    if (wgrad_partial_floats(a) > part_floats_) fail("convT_wgrad", "split-K partial buffer too small");
    const int id = prof_begin(PROF_WGRAD_SIMT, 2.0 * u.cin * u.cout * u.k * (double)x.L * x.B, st);
    conv_wgrad_simt(a, part_, st);
    colsum(dy, grads_ + u.b, false, part_, st);
    prof_end(id, st);
}

// Row-packed tensor-core operand of a ConvTranspose1d gradient: planes of dy in
// tc_yh_ / tc_yl_ (compact rows), or nullptr when the CUDA-core path applies.
const TcPlanes* Engine::convT_dy_planes(const UpP& u, const Act& dy, TcPlanes& tp, cudaStream_t st) {
    if (!convT_tc(u) || dy.L % u.s != 0) return nullptr;
    make_act_planes(dy, bw_mode(), tc_yh_, tc_yl_, st);
    tp.hi = tc_yh_; tp.lo = tc_yl_; tp.ld = tc_pitch(dy.C, bw_mode());
    if (tp.ld != dy.C) fail("convT_dgrad", "internal: row-packed planes need compact rows");
    return &tp;
}

void Engine::stats_of(const Act& x, const Stats& s, cudaStream_t st) { in_stats(x, 1e-5f, dacc_, s.mean, s.rstd, st); }

// ── AdainResBlk1d (kokoro_decoder_backward.cpp:152-285)
void Engine::blk_fwd(const BlkP& w, BlkC& c, const Act& y, cudaStream_t st) {
    const Range nvtx_range("bsml.AdainResBlk1d.fwd");
    // The leaky AdaIN outputs are cached in fp32 (the weight gradients read them)
    // and, where the next conv runs on the tensor cores, also written as its
    // operand planes in the same pass; conv1's epilogue returns norm2's statistics.
    auto planes_in = [&](void* hi, void* lo, int C, TcPlanes& tp, PlaneOut& po) {
        tp.hi = hi; tp.lo = lo; tp.ld = tc_pitch(C, tc_mode());
        po.hi = hi; po.lo = lo; po.ld = tp.ld; po.mode = tc_mode();
    };
    stats_of(c.x, c.s1, st);
    const bool tc1 = !w.up && tc_ok(w.cin, w.cout, 1);
    TcPlanes rp;
    PlaneOut ro;
    if (tc1) planes_in(tc_xh_, tc_xl_, w.cin, rp, ro);
    adain_act_fwd_v(c.x, nullptr, 1e-5f, c.s1.mean, c.s1.rstd, aff(w.n1), ACT_LEAKY, 0.2f, nullptr, &c.r,
                    tc1 ? &ro : nullptr, st);
    Act pooled = c.r;
    if (w.up) {
        dwconvT_fwd(c.r, P(w.pool_w), P(w.pool_b), 3, 2, 1, c.pooled, st);
        pooled = c.pooled;
    }
    conv(w.c1, pooled, c.c1, nullptr, 0, 1.f, false, st, tc1 ? &rp : nullptr, ssum_);
    const bool tc2 = tc_ok(w.cout, w.cout, 1);
    TcPlanes np;
    PlaneOut no;
    if (tc2) planes_in(tc_yh_, tc_yl_, w.cout, np, no);
    adain_act_fwd_v(c.c1, ssum_, 1e-5f, c.s2.mean, c.s2.rstd, aff(w.n2), ACT_LEAKY, 0.2f, nullptr, &c.n2,
                    tc2 ? &no : nullptr, st);
    // shortcut: a 1x1 conv commutes with nearest-2x, so it runs at L_in and the
    // conv2 epilogue reads it at row >> 1
    const Act* sc = &c.x;
    if (w.sc) {
        conv(w.c1x1, c.x, c.sc, nullptr, 0, 1.f, false, st);
        sc = &c.sc;
    }
    conv(w.c2, c.n2, y, sc, w.up ? 1 : 0, 1.f / std::sqrt(2.f), false, st, tc2 ? &np : nullptr);
}

void Engine::blk_bwd(const BlkP& w, BlkC& c, const Act& dY, const Act& dX, cudaStream_t st) {
    const Range nvtx_range("bsml.AdainResBlk1d.bwd");
    const int Lin = c.Lin, Lout = c.Lout;
    double* bs = grads_ ? bsum_ : nullptr;
    auto zero_bs = [&](int C) {
        if (bs) BSML_CUDA(cudaMemsetAsync(bs, 0, sizeof(double) * C, st));
    };
    auto planes_in = [&](void* hi, void* lo, int C, TcPlanes& tp, PlaneOut& po) {
        tp.hi = hi; tp.lo = lo; tp.ld = tc_pitch(C, bw_mode());
        po.hi = hi; po.lo = lo; po.ld = tp.ld; po.mode = bw_mode();
    };
    // d_branch = dY / sqrt(2) (S_[0]), in the same pass its operand planes (tc_dh_)
    // for conv2's input and weight gradients and its column sums (conv2's bias gradient)
    const bool tc2 = tc_ok(w.cout, w.cout, 1);
    Act db = view(S_[0], Lout, w.cout);
    TcPlanes dbp;
    PlaneOut dbo;
    if (tc2) planes_in(tc_dh_, tc_dl_, w.cout, dbp, dbo);
    zero_bs(w.cout);
    scale_out_v(dY, 1.f / std::sqrt(2.f), &db, tc2 ? &dbo : nullptr, bs, st);
    Act t1 = view(S_[1], Lout, w.cout);
    conv_dgrad(w.c2, db, t1, false, st, tc2 ? &dbp : nullptr);
    conv_wgrad(w.c2, db, c.n2, st, wgp(tc2 ? &dbp : nullptr), nullptr, bs);
    // dc1 (S_[2]) with its planes (tc_yh_) and column sums (conv1's bias gradient)
    const bool tc1 = tc_ok(w.cin, w.cout, 1) && tc_ok(w.cout, w.cin, 1);
    Act dc1 = view(S_[2], Lout, w.cout);
    TcPlanes dcp;
    PlaneOut dco;
    if (tc1) planes_in(tc_yh_, tc_yl_, w.cout, dcp, dco);
    zero_bs(w.cout);
    adain_act_bwd_v(c.c1, c.s2.mean, c.s2.rstd, aff(w.n2), ACT_LEAKY, 0.2f, nullptr, t1, &dc1, nullptr,
                    tc1 ? &dco : nullptr, bs, daff(w.n2), nullptr, dacc_, st);
    Act dpooled = view(S_[1], Lout, w.cin);
    conv_dgrad(w.c1, dc1, dpooled, false, st, tc1 ? &dcp : nullptr);
    conv_wgrad(w.c1, dc1, w.up ? c.pooled : c.r, st, wgp(tc1 ? &dcp : nullptr), nullptr, bs);
    Act dr = dpooled;
    if (w.up) {
        dr = view(S_[2], Lin, w.cin);
        dwconvT_dgrad(dpooled, P(w.pool_w), 3, 2, 1, dr, st);
        if (grads_) dwconvT_wgrad(dpooled, c.r, 3, 2, 1, G(w.pool_w), G(w.pool_b), dacc_, part_, st);
    }
    adain_act_bwd(c.x, c.s1.mean, c.s1.rstd, aff(w.n1), ACT_LEAKY, 0.2f, nullptr, dr, dX, nullptr, daff(w.n1),
                  nullptr, dacc_, st);
    // shortcut branch: without upsampling dbs = db and its planes are still in tc_dh_
    Act dbs = db;
    const bool tcs = w.sc && tc_ok(w.cin, w.cout, 1) && tc_ok(w.cout, w.cin, 1);
    TcPlanes sp = dbp;
    if (w.up) {
        dbs = view(S_[3], Lin, w.cout);
        pair_sum_rows(db, dbs, st);
        if (tcs) {
            make_act_planes(dbs, bw_mode(), tc_dh_, tc_dl_, st);
            sp.hi = tc_dh_; sp.lo = tc_dl_; sp.ld = tc_pitch(w.cout, bw_mode());
        }
    }
    const bool have_sp = tcs && (w.up || tc2);
    if (w.sc) {
        conv_dgrad(w.c1x1, dbs, dX, true, st, have_sp ? &sp : nullptr);
        conv_wgrad(w.c1x1, dbs, c.x, st, wgp(have_sp ? &sp : nullptr));
    } else {
        add_act(dbs, dX, 1.f, st);
    }
}

// ── AdaINResBlock1 (kokoro_decoder_backward.cpp:287-376)
// Forward: each AdaIN+Snake writes its output straight into the operand form the
// following conv reads (planes on the tensor-core path); the conv epilogue
// returns the statistics of its output for the next AdaIN.
void Engine::rb1_fwd(const RB1P& w, RB1C& c, const Act& x0, bool x0_stats, const Act& out, float out_alpha,
                     bool out_accum, cudaStream_t st) {
    const Range nvtx_range("bsml.AdaINResBlock1.fwd");
    c.x[0] = x0;
    const int L = c.L, C = w.C;
    const bool tc = tc_ok(C, C, 1);   // every conv of the block is C -> C, stride 1
    // algorithmic bytes of one AdaIN+Snake forward: read x, write y (fp32), 8 B per
    // element; the operand planes written instead of y are implementation traffic
    const double nb = 8.0 * (double)x0.numel();
    for (int i = 0; i < 3; ++i) {
        int id = prof_begin(PROF_NORM_FWD, nb, st);
        const double* sums = ssum_;   // from the previous conv's epilogue
        if (i == 0) {
            sums = nullptr;
            if (!x0_stats) {
                BSML_CUDA(cudaMemsetAsync(ssum_, 0, sizeof(double) * 2 * (size_t)B_ * C, st));
                norm_sums(x0, ssum_, st);
                sums = ssum_;
            }
        }
        const Opnd s1 = operand(tc, L, C, S_[0], tc_xh_, tc_xl_);
        adain_fwd_to(c.x[i], sums, c.st1[i], aff(w.a1[i]), ACT_SNAKE, 0.f, P(w.al1[i]), s1, st);
        prof_end(id, st);
        conv(w.c1[i], s1.f, c.c1[i], nullptr, 0, 1.f, false, st, s1.planes(), ssum_);
        id = prof_begin(PROF_NORM_FWD, nb, st);
        const Opnd s2 = operand(tc, L, C, S_[0], tc_xh_, tc_xl_);
        adain_fwd_to(c.c1[i], ssum_, c.st2[i], aff(w.a2[i]), ACT_SNAKE, 0.f, P(w.al2[i]), s2, st);
        prof_end(id, st);
        if (i < 2)
            conv(w.c2[i], s2.f, c.x[i + 1], &c.x[i], 0, 1.f, false, st, s2.planes(), ssum_);
        else
            conv(w.c2[i], s2.f, out, &c.x[i], 0, out_alpha, out_accum, st, s2.planes(), nullptr);
    }
}

// Backward: the Snake outputs (conv operands of the weight gradients) are
// recomputed from the cached inputs; each AdaIN backward writes its result as
// the operand of the next input- and weight-gradient convs and sums its
// columns for the preceding conv's bias gradient.
void Engine::rb1_bwd(const RB1P& w, RB1C& c, const Act& dOut, float scale, const Act& D, cudaStream_t st,
                     const RB1Io* io) {
    const Range nvtx_range("bsml.AdaINResBlock1.bwd");
    const int L = c.L, C = w.C;
    const bool tc = tc_ok(C, C, 1);
    const double n = (double)D.numel();
    Act t = view(S_[4], L, C);
    double* bs = grads_ ? bsum_ : nullptr;
    auto zero_bs = [&]() {
        if (bs) BSML_CUDA(cudaMemsetAsync(bs, 0, sizeof(double) * C, st));
    };
    // D = scale * dOut: fp32 (the running gradient), planes, bias sum of c2[2]; or,
    // with the entry made by the caller, planes and bias sum from there and D first
    // written by the first pair's last pass (dOut, scaled, as its skip term)
    // Under wg_split every gradient operand shared by an input and a weight gradient
    // is written twice: bw_mode() planes for the input gradient, wg_mode() ones (the
    // `_w` buffers) for the weight gradient.
    const bool split = tc && wg_split();
    Opnd Dp;
    Dp.f = D;
    if (tc) { Dp.tp.hi = tc_dh_; Dp.tp.lo = tc_dl_; Dp.tp.ld = tc_pitch(C, bw_mode()); }
    if (split) { Dp.tpw.hi = tc_dwh_; Dp.tpw.lo = tc_dwl_; Dp.tpw.ld = tc_pitch(C, wg_mode()); }
    const bool pre = io && io->in_planes;
    if (pre && !tc) fail("rb1_bwd", "internal: entry planes without the tensor-core path");
    if (pre && split && !io->in_planes_w) fail("rb1_bwd", "internal: entry planes for the weight gradient missing");
    const TcPlanes* in_planes = pre ? io->in_planes : Dp.planes();
    const TcPlanes* in_planes_w = pre ? (split ? io->in_planes_w : io->in_planes) : Dp.planes_w();
    const double* in_bs = pre ? (grads_ ? io->in_bsum : nullptr) : bs;
    if (!pre) {
        PlaneOut po, po2;
        po.hi = tc_dh_; po.lo = tc_dl_; po.ld = Dp.tp.ld; po.mode = bw_mode();
        po2.hi = tc_dwh_; po2.lo = tc_dwl_; po2.ld = Dp.tpw.ld; po2.mode = wg_mode();
        zero_bs();
        scale_out_v(dOut, scale, &D, tc ? &po : nullptr, bs, st, split ? &po2 : nullptr);
    }
    // Algorithmic bytes per element of one AdaIN+Snake backward: x and dy read, dx
    // written (fp32), 12 B, credited 8 B to the reduction pass and 4 B to the apply
    // pass; the recomputed Snake operand, the operand planes and the apply pass's
    // second read of x and dy are implementation traffic.
    for (int i = 2; i >= 0; --i) {
        const TcPlanes* dpl = i == 2 ? in_planes : Dp.planes();
        const TcPlanes* dplw = i == 2 ? in_planes_w : Dp.planes_w();
        conv_dgrad(w.c2[i], D, t, false, st, dpl);
        // s2[i] = Snake(AdaIN(c1[i])) again, as the weight-gradient operand, in the
        // same pass as the backward's reduction over (c1[i], t)
        int id = prof_begin(PROF_NORM_BWD, 8.0 * n, st);
        const Opnd s2 = operand(tc, L, C, S_[0], tc_xh_, tc_xl_, wg_mode());
        recompute_reduce_to(c.c1[i], c.st2[i], aff(w.a2[i]), ACT_SNAKE, 0.f, P(w.al2[i]), t, s2, st);
        prof_end(id, st);
        conv_wgrad(w.c2[i], D, s2.f, st, dplw, s2.planes(), i == 2 ? in_bs : bs);
        // u = gradient at conv1's output (operand of c1's dgrad and wgrad)
        id = prof_begin(PROF_NORM_BWD, 4.0 * n, st);
        Opnd u = operand(tc, L, C, S_[5], tc_yh_, tc_yl_, bw_mode());
        if (split) { u.tpw.hi = tc_uwh_; u.tpw.lo = tc_uwl_; u.tpw.ld = tc_pitch(C, wg_mode()); }
        zero_bs();
        adain_bwd_to(c.c1[i], c.st2[i], aff(w.a2[i]), ACT_SNAKE, 0.f, P(w.al2[i]), t, u, nullptr, bs, daff(w.a2[i]),
                     G(w.al2[i]), st, true);
        prof_end(id, st);
        conv_dgrad(w.c1[i], u.f, t, false, st, u.planes());
        id = prof_begin(PROF_NORM_BWD, 8.0 * n, st);
        const Opnd s1 = operand(tc, L, C, S_[0], tc_xh_, tc_xl_, wg_mode());
        recompute_reduce_to(c.x[i], c.st1[i], aff(w.a1[i]), ACT_SNAKE, 0.f, P(w.al1[i]), t, s1, st);
        prof_end(id, st);
        conv_wgrad(w.c1[i], u.f, s1.f, st, u.planes_w(), s1.planes(), bs);
        // D += gradient at this pair's input: fp32, and (except for the last pair)
        // planes and the bias sum of c2[i-1]
        Opnd Dn = Dp;
        double* bsn = nullptr;
        if (i > 0) {
            bsn = bs;
            zero_bs();
        } else {
            Dn.tp = TcPlanes{};
            Dn.tpw = TcPlanes{};
        }
        const Act* skip = &D;
        float skip_scale = 1.f;
        if (pre && i == 2) {
            skip = &dOut;
            skip_scale = scale;
        }
        bool out_accum = false;
        if (i == 0 && io && io->out) {
            Dn.f = *io->out;
            Dn.tp = io->out_planes;
            Dn.tpw = split ? io->out_planes_w : TcPlanes{};
            out_accum = io->out_accum;
            bsn = grads_ ? io->out_bsum : nullptr;
            if (bsn) BSML_CUDA(cudaMemsetAsync(bsn, 0, sizeof(double) * C, st));
        }
        id = prof_begin(PROF_NORM_BWD, 4.0 * n, st);
        adain_bwd_to(c.x[i], c.st1[i], aff(w.a1[i]), ACT_SNAKE, 0.f, P(w.al1[i]), t, Dn, skip, bsn, daff(w.a1[i]),
                     G(w.al1[i]), st, true, skip_scale, out_accum);
        prof_end(id, st);
    }
}

// ── forward
// Set-up shared by the forward entry points: the plan, copies of what the
// backward reads (F0, N, style), the packed weights and the resolved affines.
void Engine::begin_forward(int B, int T, int frames, bool have_har, int part, const float* params, const float* F0,
                           const float* N, const float* style, int style_stride, const float* aff_in,
                           float* aff_out, cudaStream_t st) {
    BSML_CUDA(cudaSetDevice(device_));
    ensure_plan(B, T, frames, have_har, part);
    const auto& cf = lay_.cfg;
    params_ = params;
    if (part != PART_GENERATOR) {
        BSML_CUDA(cudaMemcpyAsync(F0_copy_, F0, sizeof(float) * B * 2 * T, cudaMemcpyDeviceToDevice, st));
        BSML_CUDA(cudaMemcpyAsync(N_copy_, N, sizeof(float) * B * 2 * T, cudaMemcpyDeviceToDevice, st));
        F0_ = F0_copy_;
        N_ = N_copy_;
    }
    if (style)
        BSML_CUDA(cudaMemcpy2DAsync(style_copy_, sizeof(float) * cf.style_dim, style,
                                    sizeof(float) * (style_stride > 0 ? style_stride : cf.style_dim),
                                    sizeof(float) * cf.style_dim, B, cudaMemcpyDeviceToDevice, st));
    style_ = style ? style_copy_ : nullptr;
    ref_mode_ = aff_in != nullptr;
    fwd_done_ = false;
    fwd_part_ = part;
    if (part == PART_FULL && !have_har_) {
        // har is first read by the generator; the source runs on the side stream meanwhile
        BSML_CUDA(cudaEventRecord(ev_fork_, st));
        BSML_CUDA(cudaStreamWaitEvent(side_, ev_fork_, 0));
        harmonic_source(F0_copy_, B, 2 * T, cf.upsample_scale, cf.harmonic_num, cf.sample_rate, cf.n_fft, cf.hop,
                        params_ + lay_.llin_w, params_ + lay_.llin_b, hs_phase_, hs_src_, har_, side_, phase_mode_);
        BSML_CUDA(cudaEventRecord(ev_join_, side_));
    }
    pack_weights(st);
    // affines: fc(style) (compute_style_affine, kokoro_modules.cpp:563-572) or caller-supplied
    if (ref_mode_)
        BSML_CUDA(cudaMemcpyAsync(aff_, aff_in, sizeof(float) * B * lay_.aff_per_clip, cudaMemcpyDeviceToDevice, st));
    else
        affine_fc_fwd(fc_tab_, (int)lay_.aff_C.size(), fc_rows_, fc_row_entry_, params_, style_, B, cf.style_dim,
                      aff_, st);
    if (aff_out)
        BSML_CUDA(cudaMemcpyAsync(aff_out, aff_, sizeof(float) * B * lay_.aff_per_clip, cudaMemcpyDeviceToDevice, st));
}

// backbone (kokoro_decoder_backward.cpp:482-537): asr, F0_, N_ -> genin_
void Engine::run_backbone(const float* asr, cudaStream_t st) {
    const Range nvtx_range("bsml.backbone.fwd");
    const auto& cf = lay_.cfg;
    const int B = B_, T = T_;
    ncl_to_cl(asr, asr_, st);
    conv(lay_.F0c, flat_input(F0_, B, 2 * T), F0dn_, nullptr, 0, 1.f, false, st);
    conv(lay_.Nc, flat_input(N_, B, 2 * T), Ndn_, nullptr, 0, 1.f, false, st);
    conv(lay_.asr_res, asr_, asrres_, nullptr, 0, 1.f, false, st);
    copy_act(asr_, enc_in_.slice_c(0, cf.asr_dim), st);
    copy_act(F0dn_, enc_in_.slice_c(cf.asr_dim, 1), st);
    copy_act(Ndn_, enc_in_.slice_c(cf.asr_dim + 1, 1), st);
    const int nd = (int)lay_.dec.size();
    for (int i = -1; i < nd; ++i) {
        BlkC& c = i < 0 ? encc_ : decc_[i];
        const BlkP& w = i < 0 ? lay_.enc : lay_.dec[i];
        Act y;
        if (i + 1 < nd) {
            y = dec_in_[i + 1].slice_c(0, w.cout);
        } else {
            y = genin_;
        }
        blk_fwd(w, c, y, st);
        if (i + 1 < nd && res_applied_[i + 1]) {
            Act& din = dec_in_[i + 1];
            const int Cx = x_ch_[i + 1];
            copy_act(asrres_, din.slice_c(Cx, cf.asr_res_dim), st);
            copy_act(F0dn_, din.slice_c(Cx + cf.asr_res_dim, 1), st);
            copy_act(Ndn_, din.slice_c(Cx + cf.asr_res_dim + 1, 1), st);
        }
    }
}

// generator (kokoro_decoder_backward.cpp:592-667) and spectral head (:378-410): genin_, har -> audio
void Engine::run_generator(const float* har, float* audio, cudaStream_t st) {
    const Range nvtx_range("bsml.generator.fwd");
    const auto& cf = lay_.cfg;
    const int B = B_;
    if (have_har_)
        ncl_to_cl(har, har_, st);
    else
        BSML_CUDA(cudaStreamWaitEvent(st, ev_join_, 0));
    if (spk_ >= 0) {
        // the zero rows around the frames of the row-packed noise conv's input
        const int lead = lay_.noise[spk_].p, tail = spk_rows_ - lead - frames_;
        const size_t pitch_b = sizeof(float) * (size_t)har_full_.bstride;
        if (lead > 0)
            BSML_CUDA(cudaMemset2DAsync(har_full_.p, pitch_b, 0, sizeof(float) * (size_t)lead * har_full_.ld, B, st));
        if (tail > 0)
            BSML_CUDA(cudaMemset2DAsync(har_full_.p + (int64_t)(lead + frames_) * har_full_.ld, pitch_b, 0,
                                        sizeof(float) * (size_t)tail * har_full_.ld, B, st));
    }
    const int U = cf.n_ups, K = cf.n_kernels;
    for (int i = 0; i < U; ++i) {
        StageC& s = stc_[i];
        const UpP& u = lay_.ups[i];
        leaky_fwd(s.x_in, 0.1f, s.a, st);
        conv(lay_.noise[i], har_, s.xsrc, nullptr, 0, 1.f, false, st);
        rb1_fwd(lay_.nres[i], s.noise, s.xsrc, false, s.src, 1.f, false, st);
        if (i == U - 1) {
            // u written to rows 1..Lu, row 0 = reflection of row 1 (pad1d mode 1), then m = u + src
            convT(u, s.a, s.m, 1, nullptr, st);
            reflect_left1_fwd(s.m, st);
            add_act(s.src, s.m, 1.f, st);
        } else {
            convT(u, s.a, s.m, 0, &s.src, st);
        }
        for (int j = 0; j < K; ++j)
            rb1_fwd(lay_.rbs[i * K + j], s.res[j], s.m, j > 0, s.out, 1.f / (float)K, j > 0, st);
    }
    const Act& xlast = stc_[U - 1].out;
    leaky_fwd(xlast, 0.01f, xl_, st);
    conv(lay_.post, xl_, post_, nullptr, 0, 1.f, false, st);
    const int nf = cf.n_fft / 2 + 1;
    polar_fwd(post_, nf, spec_, st);
    istft_fwd(spec_, B, post_.L, cf.n_fft, cf.hop, audio, st);
}

void Engine::forward(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                     const float* style, const float* har, int frames, const float* aff_in, float* audio,
                     float* aff_out, cudaStream_t st, int style_stride) {
    const char* where = "bsml_decoder_forward";
    if (lay_.block_kind) fail(where, "the handle holds a single block: use bsml_block_forward");
    if (B < 1 || T < 1) fail(where, "B and T must be positive");
    if (style_stride != 0 && style_stride < lay_.cfg.style_dim) fail(where, "style row stride below the style width");
    if (!params || !asr || !F0 || !N || !audio) fail(where, "null input");
    if (!aff_in && !style) fail(where, "style is required unless aff_in is given");
    if (!har && lay_.cfg.har_ch != lay_.cfg.n_fft + 2)
        fail(where, "the harmonic source makes n_fft + 2 channels but har_ch = " + std::to_string(lay_.cfg.har_ch) +
                        ": pass har");
    begin_forward(B, T, frames, har != nullptr, PART_FULL, params, F0, N, style, style_stride, aff_in, aff_out, st);
    run_backbone(asr, st);
    run_generator(har, audio, st);
    fwd_done_ = true;
}

void Engine::forward_backbone(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                              const float* style, int style_stride, const float* aff_in, float* gen_in,
                              float* aff_out, cudaStream_t st) {
    const char* where = "bsml_backbone_forward";
    if (lay_.block_kind) fail(where, "the handle holds a single block");
    if (B < 1 || T < 1) fail(where, "B and T must be positive");
    if (style_stride != 0 && style_stride < lay_.cfg.style_dim) fail(where, "style row stride below the style width");
    if (!params || !asr || !F0 || !N || !gen_in) fail(where, "null input");
    if (!aff_in && !style) fail(where, "style is required unless aff_in is given");
    begin_forward(B, T, 0, false, PART_BACKBONE, params, F0, N, style, style_stride, aff_in, aff_out, st);
    run_backbone(asr, st);
    cl_to_ncl(genin_, gen_in, st);
    fwd_done_ = true;
}

void Engine::forward_generator(int B, int L_in, const float* params, const float* gen_in, const float* har,
                               int frames, const float* style, int style_stride, const float* aff_in, float* audio,
                               float* aff_out, cudaStream_t st) {
    const char* where = "bsml_generator_forward";
    if (lay_.block_kind) fail(where, "the handle holds a single block");
    if (B < 1 || L_in < 1 || frames < 2) fail(where, "B, L_in must be positive and frames at least 2");
    if (style_stride != 0 && style_stride < lay_.cfg.style_dim) fail(where, "style row stride below the style width");
    if (!params || !gen_in || !har || !audio) fail(where, "null input (the generator takes har as an input)");
    if (!aff_in && !style) fail(where, "style is required unless aff_in is given");
    begin_forward(B, L_in, frames, true, PART_GENERATOR, params, nullptr, nullptr, style, style_stride, aff_in,
                  aff_out, st);
    ncl_to_cl(gen_in, genin_, st);
    run_generator(har, audio, st);
    fwd_done_ = true;
}

int Engine::backbone_out_len(int T) const {
    int L = T;
    for (const BlkP& d : lay_.dec)
        if (d.up) L *= 2;
    return L;
}

// ── backward
void Engine::begin_backward(const char* where, int part, float* grads, cudaStream_t st) {
    if (lay_.block_kind) fail(where, "the handle holds a single block: use bsml_block_backward");
    if (!fwd_done_ || fwd_part_ != part) fail(where, "no matching forward");
    if (wg_split() && !plan_wg_) fail(where, "the math mode changed to TF32X3W after the forward");
    BSML_CUDA(cudaSetDevice(device_));
    grads_ = grads;
    if (grads_) fill(grads_, lay_.total, 0.f, st);
    // a part leaves the other part's affine gradients unwritten
    if (part != PART_FULL) fill(daff_, (int64_t)B_ * lay_.aff_per_clip, 0.f, st);
    pack_dgrad_weights(st);
}

// generator + spectral head backward; returns d(gen_in), channels-last, in S_[2] or S_[3]
Act Engine::gen_backward(const float* daudio, cudaStream_t st) {
    const Range nvtx_range("bsml.generator.bwd");
    const auto& cf = lay_.cfg;
    const int U = cf.n_ups, K = cf.n_kernels;
    // spectral head
    const int L1 = post_.L;
    const Act& xlast = stc_[U - 1].out;
    Act dpost = view(S_[0], L1, lay_.post.cout);
    istft_polar_bwd(daudio, post_, cf.n_fft, cf.hop, dpost, st);
    Act dxl = view(S_[1], L1, lay_.post.cin);
    conv_dgrad(lay_.post, dpost, dxl, false, st);
    conv_wgrad(lay_.post, dpost, xl_, st);
    // dX lives in S_[2]/S_[3] alternately; dm in S_[1]
    Act dX = view(S_[2], L1, lay_.post.cin);
    leaky_bwd(xlast, 0.01f, dxl, dX, st);
    int xbuf = 2;
    for (int i = U - 1; i >= 0; --i) {
        StageC& s = stc_[i];
        const UpP& u = lay_.ups[i];
        // dm = sum_j rb_j^T (dX / K)   (D in S_[xbuf^1], dm in S_[1])
        Act D = view(S_[xbuf ^ 1], s.Lx, u.cout);
        Act dm = view(S_[1], s.Lx, u.cout);
        if (tc_ok(u.cout, u.cout, 1)) {
            // the resblocks' common entry dX / K as planes and column sums, made once;
            // each resblock adds its input gradient into dm, the last one also writing
            // dm's planes (tc_dh_) and column sums (bsum_), the noise resblock's entry
            const int mode = bw_mode();
            PlaneOut p0;
            p0.hi = tc_eh_; p0.lo = tc_el_; p0.ld = tc_pitch(u.cout, mode); p0.mode = mode;
            TcPlanes t0;
            t0.hi = tc_eh_; t0.lo = tc_el_; t0.ld = p0.ld;
            double* bs0 = grads_ ? bsum0_ : nullptr;
            if (bs0) BSML_CUDA(cudaMemsetAsync(bs0, 0, sizeof(double) * u.cout, st));
            const bool split = wg_split();
            const int wmode = wg_mode();
            PlaneOut p0w;
            p0w.hi = tc_ewh_; p0w.lo = tc_ewl_; p0w.ld = tc_pitch(u.cout, wmode); p0w.mode = wmode;
            TcPlanes t0w;
            t0w.hi = tc_ewh_; t0w.lo = tc_ewl_; t0w.ld = p0w.ld;
            scale_out_v(dX, 1.f / (float)K, nullptr, &p0, bs0, st, split ? &p0w : nullptr);
            TcPlanes tdm, tdmw;
            tdm.hi = tc_dh_; tdm.lo = tc_dl_; tdm.ld = p0.ld;
            tdmw.hi = tc_dwh_; tdmw.lo = tc_dwl_; tdmw.ld = p0w.ld;
            for (int j = 0; j < K; ++j) {
                RB1Io io;
                io.in_planes = &t0;
                io.in_planes_w = split ? &t0w : nullptr;
                io.in_bsum = bs0;
                io.out = &dm;
                io.out_accum = j > 0;
                if (j == K - 1) {
                    io.out_planes = tdm;
                    if (split) io.out_planes_w = tdmw;
                    io.out_bsum = bsum_;
                }
                rb1_bwd(lay_.rbs[i * K + j], s.res[j], dX, 1.f / (float)K, D, st, &io);
            }
            // noise branch: affine / alpha / conv grads; its input grad only feeds noise_convs' wgrad
            RB1Io nio;
            nio.in_planes = &tdm;
            nio.in_planes_w = split ? &tdmw : nullptr;
            nio.in_bsum = bsum_;
            rb1_bwd(lay_.nres[i], s.noise, dm, 1.f, D, st, &nio);
        } else {
            for (int j = 0; j < K; ++j) {
                rb1_bwd(lay_.rbs[i * K + j], s.res[j], dX, 1.f / (float)K, D, st);
                if (j == 0) copy_act(D, dm, st);
                else add_act(D, dm, 1.f, st);
            }
            rb1_bwd(lay_.nres[i], s.noise, dm, 1.f, D, st);
        }
        conv_wgrad(lay_.noise[i], D, har_, st);
        Act du = dm;
        if (i == U - 1) {
            reflect_left1_bwd(dm, st);
            du = rows(dm, 1, s.Lu);
        }
        Act da = view(S_[xbuf ^ 1], s.Lin, u.cin);
        TcPlanes dup;
        const TcPlanes* dupp = convT_dy_planes(u, du, dup, st);
        convT_dgrad(u, du, da, st, dupp);
        convT_wgrad(u, du, s.a, st, dupp);
        Act dprev = view(S_[xbuf], s.Lin, u.cin);
        leaky_bwd(s.x_in, 0.1f, da, dprev, st);
        dX = dprev;
    }
    return dX;
}

// backbone backward (kokoro_decoder_backward.cpp:539-574) + the cat-channel grads; dY = d(gen_in) in S_[4]
void Engine::bb_backward(Act dY, cudaStream_t st) {
    const Range nvtx_range("bsml.backbone.bwd");
    const auto& cf = lay_.cfg;
    const int B = B_, T = T_;
    fill(dasrres_.p, (int64_t)B * dasrres_.bstride, 0.f, st);
    fill(dF0dn_.p, (int64_t)B * dF0dn_.bstride, 0.f, st);
    fill(dNdn_.p, (int64_t)B * dNdn_.bstride, 0.f, st);
    // the block backward uses S_[0..3]; the running dX alternates between S_[4] and S_[5]
    int ybuf = 4;
    const int nd = (int)lay_.dec.size();
    for (int i = nd - 1; i >= -1; --i) {
        BlkC& c = i < 0 ? encc_ : decc_[i];
        const BlkP& w = i < 0 ? lay_.enc : lay_.dec[i];
        Act bdx = view(S_[ybuf ^ 1], c.Lin, w.cin);
        blk_bwd(w, c, dY, bdx, st);
        if (i >= 0 && res_applied_[i]) {
            const int Cx = x_ch_[i];
            add_act(bdx.slice_c(Cx, cf.asr_res_dim), dasrres_, 1.f, st);
            add_act(bdx.slice_c(Cx + cf.asr_res_dim, 1), dF0dn_, 1.f, st);
            add_act(bdx.slice_c(Cx + cf.asr_res_dim + 1, 1), dNdn_, 1.f, st);
            dY = bdx.slice_c(0, Cx);
        } else if (i >= 0) {
            dY = bdx;
        } else {
            // encode: input = [asr, F0_dn, N_dn]
            add_act(bdx.slice_c(cf.asr_dim, 1), dF0dn_, 1.f, st);
            add_act(bdx.slice_c(cf.asr_dim + 1, 1), dNdn_, 1.f, st);
            copy_act(bdx.slice_c(0, cf.asr_dim), dasr_cl_, st);
        }
        ybuf ^= 1;
    }
    conv_wgrad(lay_.F0c, dF0dn_, flat_input(F0_, B, 2 * T), st);
    conv_wgrad(lay_.Nc, dNdn_, flat_input(N_, B, 2 * T), st);
    conv_dgrad(lay_.asr_res, dasrres_, dasr_cl_, true, st);
    conv_wgrad(lay_.asr_res, dasrres_, asr_, st);
}

// the affine outputs and the fc weight / style gradients (all AdaINs)
void Engine::finish_backward(float* d_style, float* d_aff, cudaStream_t st) {
    const auto& cf = lay_.cfg;
    const int B = B_;
    if (d_aff)
        BSML_CUDA(cudaMemcpyAsync(d_aff, daff_, sizeof(float) * B * lay_.aff_per_clip, cudaMemcpyDeviceToDevice, st));
    if (ref_mode_) {
        if (d_style) fill(d_style, (int64_t)B * cf.style_dim, 0.f, st);
    } else {
        affine_fc_bwd(fc_tab_, (int)lay_.aff_C.size(), fc_rows_, fc_row_entry_, params_, style_, daff_, B,
                      cf.style_dim, grads_, d_style, fc_part_, st);
    }
    grads_ = nullptr;
}

void Engine::backward(const float* daudio, float* grads, float* d_asr, float* d_style, float* d_aff,
                      cudaStream_t st) {
    if (!daudio) fail("bsml_decoder_backward", "null daudio");
    begin_backward("bsml_decoder_backward", PART_FULL, grads, st);
    const Act dX = gen_backward(daudio, st);
    Act dY = view(S_[4], dX.L, dX.C);
    copy_act(dX, dY, st);
    bb_backward(dY, st);
    if (d_asr) cl_to_ncl(dasr_cl_, d_asr, st);
    finish_backward(d_style, d_aff, st);
}

void Engine::backward_backbone(const float* dgen_in, float* grads, float* d_asr, float* d_style, float* d_aff,
                               cudaStream_t st) {
    if (!dgen_in) fail("bsml_backbone_backward", "null dgen_in");
    begin_backward("bsml_backbone_backward", PART_BACKBONE, grads, st);
    Act dY = view(S_[4], genin_.L, genin_.C);
    ncl_to_cl(dgen_in, dY, st);
    bb_backward(dY, st);
    if (d_asr) cl_to_ncl(dasr_cl_, d_asr, st);
    finish_backward(d_style, d_aff, st);
}

void Engine::backward_generator(const float* daudio, float* grads, float* dgen_in, float* d_style, float* d_aff,
                                cudaStream_t st) {
    if (!daudio) fail("bsml_generator_backward", "null daudio");
    begin_backward("bsml_generator_backward", PART_GENERATOR, grads, st);
    const Act dX = gen_backward(daudio, st);
    if (dgen_in) cl_to_ncl(dX, dgen_in, st);
    finish_backward(d_style, d_aff, st);
}

// ── one block (detail::adain_resblk_1d_* / adain_resblock1_*, kokoro_decoder_backward.cpp:152-376)
void Engine::forward_block(int B, int L, const float* params, const float* x, const float* style,
                           const float* aff_in, float* y, float* aff_out, cudaStream_t st) {
    if (!lay_.block_kind) fail("bsml_block_forward", "the handle holds a whole decoder: use bsml_decoder_forward");
    if (B < 1 || L < 1) fail("bsml_block_forward", "B and L must be positive");
    if (!params || !x || !y) fail("bsml_block_forward", "null input");
    if (!aff_in && !style) fail("bsml_block_forward", "style is required unless aff_in is given");
    BSML_CUDA(cudaSetDevice(device_));
    ensure_plan(B, L, 0, false, PART_FULL);
    const int S = lay_.cfg.style_dim;
    params_ = params;
    if (style) BSML_CUDA(cudaMemcpyAsync(style_copy_, style, sizeof(float) * B * S, cudaMemcpyDeviceToDevice, st));
    style_ = style ? style_copy_ : nullptr;
    ref_mode_ = aff_in != nullptr;
    fwd_done_ = false;
    pack_weights(st);
    if (ref_mode_)
        BSML_CUDA(cudaMemcpyAsync(aff_, aff_in, sizeof(float) * B * lay_.aff_per_clip, cudaMemcpyDeviceToDevice, st));
    else
        affine_fc_fwd(fc_tab_, (int)lay_.aff_C.size(), fc_rows_, fc_row_entry_, params_, style_, B, S, aff_, st);
    if (aff_out)
        BSML_CUDA(cudaMemcpyAsync(aff_out, aff_, sizeof(float) * B * lay_.aff_per_clip, cudaMemcpyDeviceToDevice, st));
    ncl_to_cl(x, blk_x_, st);
    if (lay_.block_kind == BSML_BLOCK_RESBLK1D) blk_fwd(lay_.enc, encc_, blk_y_, st);
    else rb1_fwd(lay_.rbs[0], rb1c_, blk_x_, false, blk_y_, 1.f, false, st);
    cl_to_ncl(blk_y_, y, st);
    fwd_done_ = true;
}

void Engine::backward_block(const float* dy, float* grads, float* dx, float* d_style, float* d_aff,
                            cudaStream_t st) {
    if (!lay_.block_kind) fail("bsml_block_backward", "the handle holds a whole decoder: use bsml_decoder_backward");
    if (!fwd_done_) fail("bsml_block_backward", "no matching forward");
    if (wg_split() && !plan_wg_) fail("bsml_block_backward", "the math mode changed to TF32X3W after the forward");
    if (!dy) fail("bsml_block_backward", "null dy");
    BSML_CUDA(cudaSetDevice(device_));
    const int B = B_, S = lay_.cfg.style_dim;
    grads_ = grads;
    if (grads_) fill(grads_, lay_.total, 0.f, st);
    pack_dgrad_weights(st);
    Act dX;
    if (lay_.block_kind == BSML_BLOCK_RESBLK1D) {
        // blk_bwd works in S_[0..3]
        const BlkP& w = lay_.enc;
        Act dY = view(S_[4], encc_.Lout, w.cout);
        ncl_to_cl(dy, dY, st);
        dX = view(S_[5], encc_.Lin, w.cin);
        blk_bwd(w, encc_, dY, dX, st);
    } else {
        // rb1_bwd works in S_[0], S_[4], S_[5] and D
        const RB1P& w = lay_.rbs[0];
        Act dO = view(S_[1], rb1c_.L, w.C);
        ncl_to_cl(dy, dO, st);
        dX = view(S_[2], rb1c_.L, w.C);
        rb1_bwd(w, rb1c_, dO, 1.f, dX, st);
    }
    if (dx) cl_to_ncl(dX, dx, st);
    if (d_aff)
        BSML_CUDA(cudaMemcpyAsync(d_aff, daff_, sizeof(float) * B * lay_.aff_per_clip, cudaMemcpyDeviceToDevice, st));
    if (ref_mode_) {
        if (d_style) fill(d_style, (int64_t)B * S, 0.f, st);
    } else {
        affine_fc_bwd(fc_tab_, (int)lay_.aff_C.size(), fc_rows_, fc_row_entry_, params_, style_, daff_, B, S, grads_,
                      d_style, fc_part_, st);
    }
    grads_ = nullptr;
}

}  // namespace bsml
