// safetensors reader (host side): header index, fp32 reads, and parameter
// loading by layout table with weight-norm fusion.
#pragma once

#include <cstdint>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

#include "bsml_decoder.h"

namespace bsml {

enum { ST_OTHER = 0, ST_F32 = 1, ST_F16 = 2, ST_BF16 = 3, ST_F64 = 4 };

class SafeTensors {
   public:
    struct Entry {
        std::string name;
        int dtype = ST_OTHER;
        std::vector<int64_t> shape;
        int64_t numel = 0, begin = 0, end = 0;
    };

    explicit SafeTensors(const std::string& path);
    ~SafeTensors();
    SafeTensors(const SafeTensors&) = delete;
    SafeTensors& operator=(const SafeTensors&) = delete;

    const std::vector<Entry>& entries() const { return entries_; }
    const Entry* find(const std::string& name) const;
    const std::map<std::string, std::string>& metadata() const { return meta_; }
    void read_f32(const Entry& e, float* dst) const;   // numel floats
    void load_params(const bsml_param_entry* table, int n_entries, const std::string& prefix, float* params,
                     int64_t n_params) const;

   private:
    std::string path_;
    FILE* f_ = nullptr;
    int64_t data0_ = 0;
    std::vector<Entry> entries_;
    std::map<std::string, int> index_;
    std::map<std::string, std::string> meta_;
};

}  // namespace bsml
