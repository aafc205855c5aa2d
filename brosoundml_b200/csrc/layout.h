// Flat parameter layout of the decoder (names = upstream state-dict keys under
// decoder.module.), shared by the engine and the C ABI.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "bsml_decoder.h"

namespace bsml {

struct ConvP { int64_t w = -1, b = -1; int cout = 0, cin = 0, k = 1, s = 1, p = 0, d = 1; int id = -1; };
struct AdaP { int64_t fw = -1, fb = -1; int C = 0; int idx = 0; };
struct BlkP {
    int cin = 0, cout = 0;
    bool up = false, sc = false;
    AdaP n1, n2;
    ConvP c1, c2, c1x1;
    int64_t pool_w = -1, pool_b = -1;
};
struct RB1P {
    int C = 0, k = 0;
    int dil[3] = {1, 1, 1};
    ConvP c1[3], c2[3];
    AdaP a1[3], a2[3];
    int64_t al1[3] = {-1, -1, -1}, al2[3] = {-1, -1, -1};
};
struct UpP { int64_t w = -1, b = -1; int cin = 0, cout = 0, k = 0, s = 1, p = 0; int id = -1; };

struct Layout {
    bsml_decoder_config cfg{};
    int block_kind = 0;              // 0 = full decoder, else BSML_BLOCK_* (block in enc / rbs[0])
    std::vector<bsml_param_entry> table;
    int64_t total = 0;
    ConvP F0c, Nc, asr_res;
    BlkP enc;
    std::vector<BlkP> dec;
    int64_t llin_w = -1, llin_b = -1;
    std::vector<UpP> ups;
    std::vector<ConvP> noise;
    std::vector<RB1P> nres, rbs;
    ConvP post;
    std::vector<int> aff_C;
    std::vector<int64_t> aff_base;   // per AdaIN: sum of 2*C over earlier AdaINs (per clip)
    std::vector<const AdaP*> adains; // per AdaIN index (= DecoderLora::adapters() order)
    int64_t aff_per_clip = 0;
    std::vector<ConvP*> convs;       // every regular conv (for weight packing)

    explicit Layout(const bsml_decoder_config& c);
    explicit Layout(const bsml_block_spec& b);
    Layout(const Layout&) = delete;
    Layout& operator=(const Layout&) = delete;

   private:
    void finish();   // AdaIN and conv registries
    int64_t add(const std::string& name, int nd, int s0, int s1, int s2, bool train);
    ConvP conv(const std::string& n, int cout, int cin, int k, int s, int p, int d, bool bias);
    AdaP adain(const std::string& n, int C);
    BlkP blk(const std::string& n, int cin, int cout, bool up);
    RB1P rb1(const std::string& n, int C, int k, const int* dil);
};

void validate_config(const bsml_decoder_config& c);
void validate_block(const bsml_block_spec& b);

}  // namespace bsml
