// Checkpoint reading (host side): config.json, safetensors shards and the MLX
// affine quantisation metadata, as the reference loads them
// (rucin93/qwen-mlx-runner v0.7.3, src/weights.rs, src/config.rs).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/qmr.h"

namespace qmr {

// A parsed JSON value (objects keep their key order; duplicate keys are an
// error at parse time, as the reference's strict parser requires).
struct Json {
    enum Type { Null, Bool, Number, String, Array, Object } type = Null;
    bool b = false;
    double num = 0.0;
    bool integral = false;  // a non-negative integer literal
    uint64_t u = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json *get(const std::string &key) const;
};
bool parse_json(const char *data, size_t len, Json *out, std::string *err);

// One packed or dense matrix as the reference's MatrixData::Packed holds it:
// u32 words row-major, scales and biases widened to f32.
struct HostMatrix {
    uint32_t rows = 0, cols = 0, bits = 0, group = 0;
    std::vector<uint32_t> words;
    std::vector<float> scales, biases;
};

struct QuantSpec {
    uint32_t bits = 0, group = 0;
};

class Checkpoint {
public:
    ~Checkpoint();
    // Checkpoint::open (src/weights.rs:53-289): config.json, one
    // .safetensors file or an index with shards, canonical tensor names.
    static int open(const std::string &dir, std::unique_ptr<Checkpoint> *out);
    // Checkpoint::matrix (src/weights.rs:292-351).
    int matrix(const std::string &name, HostMatrix *m) const;
    // Checkpoint::vector (src/weights.rs:353-368): rank-1 float tensor, +1 for
    // zero-centred norms of a raw Hugging Face checkpoint.
    int vector(const std::string &name, std::vector<float> *v) const;
    // Checkpoint::conv (src/weights.rs:370-389).
    int conv(const std::string &name, uint32_t channels, uint32_t width, std::vector<float> *v) const;
    bool contains(const std::string &name) const;
    const QmrModelConfig &config() const { return cfg_; }
    uint32_t max_position() const { return max_pos_; }
    bool tied() const { return tied_; }

private:
    struct Tensor {
        int file = 0;
        size_t offset = 0, length = 0;
        std::vector<uint64_t> shape;
        std::string dtype;
        bool raw_hf = false;
    };
    struct Mapping {
        void *base = nullptr;
        size_t len = 0;
    };
    int parse_file(const std::string &path, int file_id, std::map<std::string, Tensor> *entries);
    int floats(const Tensor &t, std::vector<float> *out) const;
    const Tensor *tensor(const std::string &key) const;
    const uint8_t *bytes(const Tensor &t) const;

    QmrModelConfig cfg_{};
    uint32_t max_pos_ = 0;
    bool tied_ = false;
    bool has_default_quant_ = false;
    QuantSpec default_quant_;
    std::map<std::string, std::pair<bool, QuantSpec>> quant_overrides_;  // module -> (quantised?, spec)
    std::vector<Mapping> files_;
    std::map<std::string, Tensor> tensors_;
};

// ModelConfig::from_json + validate (src/config.rs:29-235).
int model_config_from_json(const Json &root, QmrModelConfig *cfg, uint32_t *max_position, bool *tied);

}  // namespace qmr
