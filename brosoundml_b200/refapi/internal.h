// Internals of the reference-signature C++ layer (libbsml_ref.so): shared helpers
// over the C ABI of libbsml_b200.so. This layer makes no CUDA call of its own.
#pragma once

#include <brotensor/tensor.h>

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "bsml_decoder.h"
#include "brosoundml/kokoro_modules.h"

namespace brosoundml {
namespace refapi {

// a failed C-ABI call re-raised with its message ("brosoundml: <where>: <reason>")
inline void check(int rc) {
    if (rc != 0) throw std::runtime_error(bsml_last_error());
}
// for the calls that return a count on success (bsml_*_param_table)
inline int check_count(int rc) {
    if (rc < 0) throw std::runtime_error(bsml_last_error());
    return rc;
}
[[noreturn]] inline void fail(const std::string& where, const std::string& why) {
    throw std::runtime_error("brosoundml: " + where + ": " + why);
}
inline void need(bool ok, const char* where, const std::string& why) {
    if (!ok) fail(where, why);
}
inline void sync() { check(bsml_synchronize()); }

// device-side copy of n floats (any device-reachable addresses)
inline void copy_floats(float* dst, const float* src, std::int64_t n) {
    if (n > 0) check(bsml_memcpy(dst, src, n * (std::int64_t)sizeof(float), nullptr));
}

// The flat parameter vector of a decoder or block handle, filled by name from
// the reference's weight structs on every call.
class ParamBuf {
   public:
    ParamBuf() = default;
    ~ParamBuf();
    ParamBuf(const ParamBuf&) = delete;
    ParamBuf& operator=(const ParamBuf&) = delete;
    void init(const bsml_decoder* h);
    // copies t into the named tensor; an empty t (a disabled bias) writes zeros.
    // Throws when the name is unknown or the sizes differ.
    void set(const std::string& name, const brotensor::Tensor& t, const char* where);
    float* data() const { return p_; }
    std::int64_t size() const { return n_; }

   private:
    const bsml_param_entry* find(const std::string& name) const;
    std::vector<bsml_param_entry> table_;
    float* p_ = nullptr;
    float* zeros_ = nullptr;
    std::int64_t n_ = 0, max_entry_ = 0;
};

// A GPU engine handle (whole decoder or one block) with its parameter vector and
// a packed-affine buffer; what a forward cache's `state` holds.
struct EngineState {
    bsml_decoder* h = nullptr;
    std::vector<unsigned char> key;   // the config / spec it was built for
    ParamBuf params;
    float* aff = nullptr;             // (aff_per_clip) packed (gamma ; beta) per AdaIN
    float* daff = nullptr;
    std::int64_t aff_per_clip = 0;
    std::vector<int> aff_C;
    int part_T = 0;                   // T (backbone) or L_in (generator) of the last forward
    ~EngineState();
};

// The engine for a config (reused when `cur` was built for the same one).
std::shared_ptr<EngineState> decoder_state(const bsml_decoder_config& cfg, std::shared_ptr<void> cur);
std::shared_ptr<EngineState> block_state(const bsml_block_spec& spec, std::shared_ptr<void> cur);

// Architecture of the reference's structs. A part that is absent (no generator
// for a backbone-only call, no backbone for a generator-only call) gets a small
// stand-in that is never run.
bsml_decoder_config config_of(const DecoderBackbone* bb, const Generator* gen);
bsml_block_spec spec_of(const AdainResBlk1dWeights& w);
bsml_block_spec spec_of(const AdaINResBlock1Weights& w);

// Parameter filling by the layout's (upstream) names.
void fill_block(ParamBuf& P, const std::string& prefix, const AdainResBlk1dWeights& w, const char* where);
void fill_rb1(ParamBuf& P, const std::string& prefix, const AdaINResBlock1Weights& w, const char* where);
void fill_backbone(ParamBuf& P, const DecoderBackbone& bb, const char* where);
void fill_generator(ParamBuf& P, const Generator& gen, const char* where);

// out reshaped to (r, c) with the device tag of `like`
void shape_out(brotensor::Tensor& out, int r, int c, const brotensor::Tensor& like);
// t must hold n elements
void need_size(const brotensor::Tensor& t, std::int64_t n, const char* where, const char* what);

}  // namespace refapi
}  // namespace brosoundml
