// Conv1d weight gradient for callers that cannot allocate device memory.
//
// Some callers may not call cudaMalloc on the path that computes gradients: a
// real-time audio host (a plugin's processing thread must never block on the
// driver's allocator), or an embedding application whose device memory is all
// reserved up front by its own arena. For them this entry point takes its
// scratch — channels-last copies of dy and x plus the split-K partial sums —
// from one file-scope device array of fixed size instead of allocating.
#include <cstdint>
#include <mutex>
#include <string>

#include "bsml_decoder.h"
#include "kernels.h"

namespace {

// 4 Mi floats = 16 MiB, held by every GPU that loads the library until exit.
constexpr int64_t kScratchFloats = BSML_NOALLOC_SCRATCH_FLOATS;
__device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (cudaGetSymbolAddress, with that device current) and cached.
float* scratch_on_current_device() {
    int dev = 0;
    bsml::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) bsml::fail("bsml_conv1d_backward_weight_noalloc", "device index out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        bsml::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress");
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    return g_scratch_ptr[dev];
}

int64_t r64(int64_t n) { return bsml::round_up(n, 64); }

}  // namespace

extern "C" int bsml_conv1d_backward_weight_noalloc(const float* dy, const float* x, int B, int Ci, int L, int Co,
                                                    int k, int stride, int pad, int dil, float* dW, float* db,
                                                    void* stream) {
    try {
        const char* where = "bsml_conv1d_backward_weight_noalloc";
        // a padded input shorter than the dilated kernel has no output (the numerator
        // is negative; C division would truncate it to an output of length 1)
        const int64_t num = (int64_t)L + 2 * (int64_t)pad - (int64_t)dil * (k - 1) - 1;
        const int Lo = (num < 0 || stride <= 0) ? 0 : (int)(num / stride + 1);
        if (!dy || !x || !dW || B <= 0 || Ci <= 0 || Co <= 0 || k <= 0 || stride <= 0 || dil <= 0 || Lo <= 0)
            bsml::fail(where, "bad argument");
        bsml::Act ga, xa;
        ga.B = B; ga.L = Lo; ga.C = Co; ga.ld = bsml::pitch(Co); ga.bstride = (int64_t)Lo * ga.ld;
        xa.B = B; xa.L = L; xa.C = Ci; xa.ld = bsml::pitch(Ci); xa.bstride = (int64_t)L * xa.ld;
        const int64_t n_dy = r64((int64_t)B * ga.bstride), n_x = r64((int64_t)B * xa.bstride);
        const int64_t wsize = (int64_t)Co * Ci * k;
        const int64_t need = n_dy + n_x + std::max<int64_t>(wsize, Co);   // one split at least
        if (need > kScratchFloats)
            bsml::fail(where, "problem needs " + std::to_string(need) + " floats of scratch; the static maximum is " +
                                  std::to_string(kScratchFloats) + " floats (" +
                                  std::to_string(kScratchFloats * 4 >> 20) + " MiB)");
        float* s = scratch_on_current_device();
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        ga.p = s;
        xa.p = s + n_dy;
        float* part = s + n_dy + n_x;
        bsml::ncl_to_cl(dy, ga, st);
        bsml::ncl_to_cl(x, xa, st);
        bsml::ConvWgrad a;
        a.dy = ga; a.x = xa; a.k = k; a.s = stride; a.p = pad; a.d = dil; a.dW = dW; a.db = db;
        if (!bsml::conv_wgrad_simt_capped(a, part, kScratchFloats - n_dy - n_x, st))
            bsml::fail(where, "scratch too small for one split");
        return 0;
    } catch (const std::exception& e) {
        bsml::set_last_error(e.what());
        return -1;
    }
}
