// Checkpoint reading: a strict JSON parser, safetensors shards (memory
// mapped), the MLX affine quantisation metadata and the model configuration.
//
// The accepted formats and checks restate the reference's loader
// (rucin93/qwen-mlx-runner v0.7.3): src/weights.rs (Checkpoint::open,
// matrix, vector, conv, parse_safetensors, parse_quantization,
// canonical_name, weight_key) and src/config.rs (ModelConfig::from_json,
// validate).  The names and rules have to match: they define which
// checkpoints load and how their tensors map onto the model.
#include "checkpoint.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <dirent.h>
#include <fstream>
#include <set>
#include <sstream>

#include "qmr_internal.h"

namespace qmr {

// ---- JSON ------------------------------------------------------------------

const Json *Json::get(const std::string &key) const {
    if (type != Object) return nullptr;
    for (const auto &kv : obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

namespace {

struct JsonParser {
    const char *p, *end;
    std::string err;
    int depth = 0;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail_at(const char *msg) {
        if (err.empty()) err = msg;
        return false;
    }
    bool literal(const char *lit) {
        const size_t n = strlen(lit);
        if ((size_t)(end - p) < n || memcmp(p, lit, n) != 0) return fail_at("invalid JSON literal");
        p += n;
        return true;
    }
    static void utf8(std::string &s, uint32_t cp) {
        if (cp < 0x80) {
            s += (char)cp;
        } else if (cp < 0x800) {
            s += (char)(0xC0 | (cp >> 6));
            s += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            s += (char)(0xE0 | (cp >> 12));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        } else {
            s += (char)(0xF0 | (cp >> 18));
            s += (char)(0x80 | ((cp >> 12) & 0x3F));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(uint32_t *v) {
        if (end - p < 4) return fail_at("truncated \\u escape");
        *v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p++;
            *v <<= 4;
            if (c >= '0' && c <= '9')
                *v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f')
                *v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F')
                *v |= (uint32_t)(c - 'A' + 10);
            else
                return fail_at("invalid \\u escape");
        }
        return true;
    }
    bool string(std::string *out) {
        if (p >= end || *p != '"') return fail_at("expected a JSON string");
        ++p;
        out->clear();
        while (p < end && *p != '"') {
            const char c = *p++;
            if ((unsigned char)c < 0x20) return fail_at("control character in JSON string");
            if (c != '\\') {
                *out += c;
                continue;
            }
            if (p >= end) return fail_at("truncated JSON escape");
            const char e = *p++;
            switch (e) {
                case '"': *out += '"'; break;
                case '\\': *out += '\\'; break;
                case '/': *out += '/'; break;
                case 'b': *out += '\b'; break;
                case 'f': *out += '\f'; break;
                case 'n': *out += '\n'; break;
                case 'r': *out += '\r'; break;
                case 't': *out += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {
                        uint32_t lo;
                        if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail_at("unpaired surrogate");
                        p += 2;
                        if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return fail_at("invalid surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return fail_at("unpaired surrogate");
                    }
                    utf8(*out, cp);
                    break;
                }
                default: return fail_at("invalid JSON escape");
            }
        }
        if (p >= end) return fail_at("unterminated JSON string");
        ++p;
        return true;
    }
    bool number(Json *v) {
        const char *s = p;
        if (p < end && *p == '-') ++p;
        bool digits = false, plain = true;
        while (p < end && *p >= '0' && *p <= '9') ++p, digits = true;
        if (p < end && *p == '.') {
            plain = false;
            ++p;
            while (p < end && *p >= '0' && *p <= '9') ++p;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            plain = false;
            ++p;
            if (p < end && (*p == '+' || *p == '-')) ++p;
            while (p < end && *p >= '0' && *p <= '9') ++p;
        }
        if (!digits) return fail_at("invalid JSON number");
        const std::string text(s, p);
        v->type = Json::Number;
        v->num = strtod(text.c_str(), nullptr);
        if (!std::isfinite(v->num)) return fail_at("non-finite JSON number");
        v->integral = plain && text[0] != '-';
        if (v->integral) {
            errno = 0;
            v->u = strtoull(text.c_str(), nullptr, 10);
            if (errno == ERANGE) v->integral = false;
        }
        return true;
    }
    bool value(Json *v) {
        if (++depth > 128) return fail_at("JSON nested too deeply");
        ws();
        if (p >= end) return fail_at("unexpected end of JSON");
        bool ok = true;
        const char c = *p;
        if (c == '{') {
            ++p;
            v->type = Json::Object;
            ws();
            if (p < end && *p == '}') {
                ++p;
            } else {
                std::set<std::string> seen;
                for (;;) {
                    ws();
                    std::string key;
                    if (!string(&key)) return false;
                    if (!seen.insert(key).second) return fail_at("duplicate JSON key");
                    ws();
                    if (p >= end || *p != ':') return fail_at("expected ':' in JSON object");
                    ++p;
                    Json item;
                    if (!value(&item)) return false;
                    v->obj.emplace_back(std::move(key), std::move(item));
                    ws();
                    if (p < end && *p == ',') {
                        ++p;
                        continue;
                    }
                    if (p < end && *p == '}') {
                        ++p;
                        break;
                    }
                    return fail_at("expected ',' or '}' in JSON object");
                }
            }
        } else if (c == '[') {
            ++p;
            v->type = Json::Array;
            ws();
            if (p < end && *p == ']') {
                ++p;
            } else {
                for (;;) {
                    Json item;
                    if (!value(&item)) return false;
                    v->arr.push_back(std::move(item));
                    ws();
                    if (p < end && *p == ',') {
                        ++p;
                        continue;
                    }
                    if (p < end && *p == ']') {
                        ++p;
                        break;
                    }
                    return fail_at("expected ',' or ']' in JSON array");
                }
            }
        } else if (c == '"') {
            v->type = Json::String;
            ok = string(&v->str);
        } else if (c == 't') {
            v->type = Json::Bool;
            v->b = true;
            ok = literal("true");
        } else if (c == 'f') {
            v->type = Json::Bool;
            ok = literal("false");
        } else if (c == 'n') {
            v->type = Json::Null;
            ok = literal("null");
        } else {
            ok = number(v);
        }
        --depth;
        return ok;
    }
};

}  // namespace

bool parse_json(const char *data, size_t len, Json *out, std::string *err) {
    JsonParser jp{data, data + len, {}, 0};
    *out = Json();
    if (!jp.value(out)) {
        if (err) *err = jp.err;
        return false;
    }
    jp.ws();
    if (jp.p != jp.end) {
        if (err) *err = "trailing data after JSON value";
        return false;
    }
    return true;
}

// ---- model configuration -----------------------------------------------------

namespace {

bool read_file(const std::string &path, std::string *out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    *out = ss.str();
    return true;
}

bool get_uint(const Json &t, const char *key, uint32_t *v) {
    const Json *j = t.get(key);
    if (j == nullptr || j->type != Json::Number || !j->integral || j->u > 0xffffffffull) return false;
    *v = (uint32_t)j->u;
    return true;
}

bool get_num(const Json *j, double *v) {
    if (j == nullptr || j->type != Json::Number) return false;
    *v = j->num;
    return true;
}

// canonical_name (src/weights.rs:457-472).
std::string canonical_name(const std::string &name) {
    auto starts = [&](const char *pfx) { return name.rfind(pfx, 0) == 0; };
    if (starts("model.language_model.")) return "model." + name.substr(strlen("model.language_model."));
    if (starts("language_model.model.")) return "model." + name.substr(strlen("language_model.model."));
    if (starts("language_model.")) {
        const std::string rest = name.substr(strlen("language_model."));
        return rest.rfind("lm_head", 0) == 0 ? rest : "model." + rest;
    }
    return name;
}

bool ends_with(const std::string &s, const char *suffix) {
    const size_t n = strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

// weight_key (src/weights.rs:474-486).
std::string weight_key(const std::string &name) {
    const std::string key = canonical_name(name);
    if (ends_with(key, ".weight") || ends_with(key, ".scales") || ends_with(key, ".biases") ||
        ends_with(key, ".A_log") || ends_with(key, ".dt_bias"))
        return key;
    return key + ".weight";
}

// is_zero_centered_norm (src/weights.rs:488-494).
bool zero_centered_norm(const std::string &key) {
    return key == "model.norm.weight" || ends_with(key, ".input_layernorm.weight") ||
           ends_with(key, ".post_attention_layernorm.weight") || ends_with(key, ".q_norm.weight") ||
           ends_with(key, ".k_norm.weight");
}

// parse_quant_spec (src/weights.rs:711-738).
int parse_quant_spec(const Json &v, QuantSpec *q) {
    const Json *mode = v.get("mode");
    if (mode != nullptr && (mode->type != Json::String || mode->str != "affine"))
        return fail(QMR_EUNSUPPORTED, "unsupported quantization mode");
    uint32_t bits = 0, group = 0;
    if (!get_uint(v, "bits", &bits)) return fail(QMR_EINVAL, "missing quantization bits");
    if (bits != 4 && bits != 8) return fail(QMR_EUNSUPPORTED, "unsupported quantization bit width %u", bits);
    if (!get_uint(v, "group_size", &group)) return fail(QMR_EINVAL, "missing quantization group size");
    if (group == 0 || group % (32 / bits) != 0) return fail(QMR_EINVAL, "invalid quantization group size");
    q->bits = bits;
    q->group = group;
    return QMR_OK;
}

uint16_t f16_bits_le(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// IEEE binary16 -> f32, exact (the widening half::f16::to_f32 performs).
float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

int model_config_from_json(const Json &root, QmrModelConfig *cfg, uint32_t *max_position, bool *tied) {
    if (root.type != Json::Object) return fail(QMR_EINVAL, "config.json is not an object");
    const Json *tc = root.get("text_config");
    const Json &t = tc != nullptr ? *tc : root;
    const Json *mt = root.get("model_type");
    const Json *tt = t.get("model_type");
    const std::string model_type = mt && mt->type == Json::String ? mt->str : "";
    const std::string text_type = tt && tt->type == Json::String ? tt->str : "";
    if (!((model_type == "qwen3_5" || model_type == "qwen3_5_text") && (text_type == "qwen3_5_text" || text_type.empty())))
        return fail(QMR_EUNSUPPORTED, "unsupported model architecture: %s/%s", model_type.c_str(), text_type.c_str());
    for (const char *moe : {"num_experts", "num_local_experts", "moe_intermediate_size", "shared_expert_intermediate_size"})
        if (t.get(moe) != nullptr) return fail(QMR_EUNSUPPORTED, "MoE field %s is unsupported", moe);
    const Json *rs = t.get("rope_scaling");
    if (rs != nullptr && rs->type != Json::Null) return fail(QMR_EUNSUPPORTED, "RoPE scaling is unsupported");
    const Json *ab = t.get("attention_bias");
    if (ab != nullptr && !(ab->type == Json::Bool && !ab->b))
        return fail(QMR_EUNSUPPORTED, "text_config.attention_bias must be false");
    const Json *act = t.get("hidden_act");
    if (act != nullptr && !(act->type == Json::String && act->str == "silu"))
        return fail(QMR_EUNSUPPORTED, "text_config.hidden_act must be silu");
    const Json *rope = t.get("rope_parameters");
    if (rope != nullptr) {
        const Json *rt = rope->get("rope_type");
        if (rt != nullptr && !(rt->type == Json::String && rt->str == "default"))
            return fail(QMR_EUNSUPPORTED, "unsupported RoPE type");
        if (rope->get("factor") != nullptr) return fail(QMR_EUNSUPPORTED, "RoPE scaling is unsupported");
    }
    QmrModelConfig c{};
    uint32_t interval = 0, maxpos = 0;
    struct {
        const char *key;
        uint32_t *dst;
    } fields[] = {{"hidden_size", &c.hidden_size},
                  {"intermediate_size", &c.intermediate_size},
                  {"num_hidden_layers", &c.num_layers},
                  {"num_attention_heads", &c.num_heads},
                  {"num_key_value_heads", &c.num_kv_heads},
                  {"head_dim", &c.head_dim},
                  {"vocab_size", &c.vocab_size},
                  {"linear_num_key_heads", &c.linear_key_heads},
                  {"linear_num_value_heads", &c.linear_value_heads},
                  {"linear_key_head_dim", &c.linear_key_dim},
                  {"linear_value_head_dim", &c.linear_value_dim},
                  {"linear_conv_kernel_dim", &c.conv_width},
                  {"full_attention_interval", &interval},
                  {"max_position_embeddings", &maxpos}};
    for (auto &f : fields) {
        if (!get_uint(t, f.key, f.dst)) return fail(QMR_EINVAL, "missing or invalid text_config.%s", f.key);
        if (*f.dst == 0) return fail(QMR_EINVAL, "%s must be positive", f.key);
    }
    double eps = 0, theta = 0, partial = 0;
    if (!get_num(t.get("rms_norm_eps"), &eps)) return fail(QMR_EINVAL, "missing or invalid text_config.rms_norm_eps");
    const Json *th = rope != nullptr && rope->get("rope_theta") ? rope->get("rope_theta") : t.get("rope_theta");
    if (!get_num(th, &theta)) return fail(QMR_EINVAL, "missing RoPE theta");
    const Json *pf = rope != nullptr && rope->get("partial_rotary_factor") ? rope->get("partial_rotary_factor")
                                                                          : t.get("partial_rotary_factor");
    if (!get_num(pf, &partial)) return fail(QMR_EINVAL, "missing partial rotary factor");
    c.rms_eps = (float)eps;
    c.rope_theta = (float)theta;
    if (!(std::isfinite(c.rms_eps) && c.rms_eps > 0)) return fail(QMR_EINVAL, "invalid RMS epsilon");
    if (!(std::isfinite(c.rope_theta) && c.rope_theta > 0)) return fail(QMR_EINVAL, "invalid RoPE theta");
    const float pr = (float)partial;
    if (!(std::isfinite(pr) && pr > 0 && pr <= 1)) return fail(QMR_EINVAL, "invalid partial rotary factor");
    c.rotary_dim = (uint32_t)((double)c.head_dim * (double)pr);
    if (c.rotary_dim == 0 || c.rotary_dim % 2 != 0 || c.rotary_dim > c.head_dim)
        return fail(QMR_EINVAL, "partial rotary dimension must be even and fit head");
    if (c.num_heads % c.num_kv_heads != 0) return fail(QMR_EINVAL, "attention heads must divide into KV heads");
    if (c.num_layers > QMR_MAX_LAYERS) return fail(QMR_EUNSUPPORTED, "more than %d layers", QMR_MAX_LAYERS);
    const Json *lt = t.get("layer_types");
    if (lt == nullptr || lt->type != Json::Array) return fail(QMR_EINVAL, "missing text_config.layer_types");
    if (lt->arr.size() != c.num_layers) return fail(QMR_EINVAL, "layer count mismatch");
    for (uint32_t i = 0; i < c.num_layers; ++i) {
        const Json &k = lt->arr[i];
        if (k.type != Json::String) return fail(QMR_EINVAL, "invalid layer type");
        const char *expected = (i + 1) % interval == 0 ? "full_attention" : "linear_attention";
        if (k.str != expected) return fail(QMR_EINVAL, "layer %u must be %s, got %s", i, expected, k.str.c_str());
        c.is_attention[i] = (i + 1) % interval == 0 ? 1 : 0;
    }
    bool tie = false;
    const Json *tw = t.get("tie_word_embeddings");
    if (tw == nullptr) tw = root.get("tie_word_embeddings");
    if (tw != nullptr && tw->type == Json::Bool) tie = tw->b;
    *cfg = c;
    *max_position = maxpos;
    *tied = tie;
    return QMR_OK;
}

// ---- safetensors ---------------------------------------------------------------

Checkpoint::~Checkpoint() {
    for (auto &m : files_)
        if (m.base != nullptr) munmap(m.base, m.len);
}

// parse_safetensors (src/weights.rs:569-677): header length, strict JSON
// header, known dtypes, positive dimensions, byte lengths matching the
// shapes, data ranges that tile the body with no overlap or hole.
int Checkpoint::parse_file(const std::string &path, int file_id, std::map<std::string, Tensor> *entries) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail(QMR_EINVAL, "open %s failed", path.c_str());
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        return fail(QMR_EINVAL, "stat %s failed", path.c_str());
    }
    const size_t len = (size_t)st.st_size;
    void *base = len > 0 ? mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    ::close(fd);
    if (len > 0 && base == MAP_FAILED) return fail(QMR_EINVAL, "map %s failed", path.c_str());
    files_.push_back({base, len});
    const uint8_t *m = static_cast<const uint8_t *>(base);
    if (len < 8) return fail(QMR_EINVAL, "safetensors header truncated");
    uint64_t hlen = 0;
    memcpy(&hlen, m, 8);
    if (hlen > 100000000ull) return fail(QMR_EINVAL, "safetensors header exceeds 100 MB");
    if (8 + hlen > len) return fail(QMR_EINVAL, "safetensors header truncated");
    Json header;
    std::string err;
    if (!parse_json(reinterpret_cast<const char *>(m + 8), (size_t)hlen, &header, &err))
        return fail(QMR_EINVAL, "invalid safetensors JSON header: %s", err.c_str());
    if (header.type != Json::Object) return fail(QMR_EINVAL, "safetensors header is not an object");
    const size_t data_start = 8 + (size_t)hlen;
    std::vector<std::pair<size_t, size_t>> ranges;
    for (const auto &kv : header.obj) {
        const std::string &name = kv.first;
        const Json &v = kv.second;
        if (name == "__metadata__") {
            if (v.type != Json::Object) return fail(QMR_EINVAL, "invalid safetensors metadata");
            for (const auto &mkv : v.obj)
                if (mkv.second.type != Json::String) return fail(QMR_EINVAL, "invalid safetensors metadata value");
            continue;
        }
        const Json *dt = v.get("dtype");
        if (dt == nullptr || dt->type != Json::String) return fail(QMR_EINVAL, "%s: missing dtype", name.c_str());
        size_t item = 0;
        const std::string &d = dt->str;
        if (d == "F16" || d == "BF16")
            item = 2;
        else if (d == "F32" || d == "U32" || d == "I32")
            item = 4;
        else if (d == "F64" || d == "I64" || d == "U64")
            item = 8;
        else if (d == "U8" || d == "I8" || d == "BOOL")
            item = 1;
        else
            return fail(QMR_EINVAL, "%s: unsupported dtype %s", name.c_str(), d.c_str());
        const Json *sh = v.get("shape");
        if (sh == nullptr || sh->type != Json::Array) return fail(QMR_EINVAL, "%s: missing shape", name.c_str());
        Tensor t;
        t.file = file_id;
        t.dtype = d;
        uint64_t count = 1;
        for (const Json &dim : sh->arr) {
            if (dim.type != Json::Number || !dim.integral) return fail(QMR_EINVAL, "invalid tensor dimension");
            if (dim.u == 0) return fail(QMR_EINVAL, "zero tensor dimension");
            if (count > UINT64_MAX / dim.u) return fail(QMR_ERANGE, "%s: tensor element count overflow", name.c_str());
            count *= dim.u;
            t.shape.push_back(dim.u);
        }
        if (count > UINT64_MAX / item) return fail(QMR_ERANGE, "%s: tensor byte length overflow", name.c_str());
        const uint64_t nbytes = count * item;
        const Json *off = v.get("data_offsets");
        if (off == nullptr || off->type != Json::Array || off->arr.size() != 2 || off->arr[0].type != Json::Number ||
            !off->arr[0].integral || off->arr[1].type != Json::Number || !off->arr[1].integral)
            return fail(QMR_EINVAL, "%s: invalid data offsets", name.c_str());
        const uint64_t a = off->arr[0].u, b = off->arr[1].u;
        if (b < a || b - a != nbytes) return fail(QMR_EINVAL, "%s: byte length mismatch", name.c_str());
        if (data_start + b > len) return fail(QMR_EINVAL, "%s: tensor exceeds file", name.c_str());
        t.offset = data_start + (size_t)a;
        t.length = (size_t)nbytes;
        ranges.emplace_back((size_t)a, (size_t)b);
        (*entries)[name] = t;
    }
    std::sort(ranges.begin(), ranges.end());
    size_t until = 0;
    for (const auto &r : ranges) {
        if (r.first != until) return fail(QMR_EINVAL, "safetensors data ranges overlap or leave holes");
        until = r.second;
    }
    if (until != len - data_start) return fail(QMR_EINVAL, "safetensors data has unindexed trailing bytes");
    return QMR_OK;
}

int Checkpoint::open(const std::string &dir, std::unique_ptr<Checkpoint> *out) {
    std::unique_ptr<Checkpoint> cp(new Checkpoint());
    std::string text;
    if (!read_file(dir + "/config.json", &text)) return fail(QMR_EINVAL, "read checkpoint config.json failed");
    Json root;
    std::string err;
    if (!parse_json(text.data(), text.size(), &root, &err)) return fail(QMR_EINVAL, "invalid config.json: %s", err.c_str());
    int rc = model_config_from_json(root, &cp->cfg_, &cp->max_pos_, &cp->tied_);
    if (rc != QMR_OK) return rc;
    // parse_quantization (src/weights.rs:679-709).
    const Json *qv = root.get("quantization");
    if (qv == nullptr) qv = root.get("quantization_config");
    if (qv != nullptr) {
        if (qv->type != Json::Object) return fail(QMR_EINVAL, "invalid quantization metadata");
        if (qv->get("bits") != nullptr || qv->get("group_size") != nullptr) {
            rc = parse_quant_spec(*qv, &cp->default_quant_);
            if (rc != QMR_OK) return rc;
            cp->has_default_quant_ = true;
        }
        for (const auto &kv : qv->obj) {
            if (kv.first == "bits" || kv.first == "group_size" || kv.first == "mode") continue;
            std::pair<bool, QuantSpec> spec{false, {}};
            if (kv.second.type == Json::Bool) {
                if (kv.second.b) {
                    spec.first = cp->has_default_quant_;
                    spec.second = cp->default_quant_;
                }
            } else if (kv.second.type == Json::Object) {
                rc = parse_quant_spec(kv.second, &spec.second);
                if (rc != QMR_OK) return rc;
                spec.first = true;
            } else {
                return fail(QMR_EINVAL, "invalid quantization entry %s", kv.first.c_str());
            }
            if (!cp->quant_overrides_.emplace(canonical_name(kv.first), spec).second)
                return fail(QMR_EINVAL, "duplicate quantization entry %s", kv.first.c_str());
        }
    }
    // One .safetensors file, or the shards an index names.
    std::vector<std::string> files;
    std::map<std::string, std::string> weight_map;
    std::string index;
    const bool indexed = read_file(dir + "/model.safetensors.index.json", &index);
    if (indexed) {
        Json ij;
        if (!parse_json(index.data(), index.size(), &ij, &err)) return fail(QMR_EINVAL, "invalid safetensors index");
        const Json *wm = ij.get("weight_map");
        if (wm == nullptr || wm->type != Json::Object) return fail(QMR_EINVAL, "missing safetensors weight_map");
        if (wm->obj.empty()) return fail(QMR_EINVAL, "empty safetensors index");
        std::set<std::string> names;
        for (const auto &kv : wm->obj) {
            if (kv.second.type != Json::String) return fail(QMR_EINVAL, "invalid shard filename");
            const std::string &f = kv.second.str;
            if (f.find('/') != std::string::npos || f == "." || f == ".." || !ends_with(f, ".safetensors"))
                return fail(QMR_EINVAL, "unsafe shard filename %s", f.c_str());
            names.insert(f);
            weight_map[kv.first] = f;
        }
        files.assign(names.begin(), names.end());
    } else {
        DIR *d = opendir(dir.c_str());
        if (d == nullptr) return fail(QMR_EINVAL, "checkpoint path must be a directory");
        while (dirent *e = readdir(d)) {
            const std::string n = e->d_name;
            if (ends_with(n, ".safetensors")) files.push_back(n);
        }
        closedir(d);
        std::sort(files.begin(), files.end());
        if (files.size() != 1) return fail(QMR_EINVAL, "expected one safetensors file or an index");
    }
    std::set<std::string> seen;
    int conv_layout = -1;  // 1: HF [channels, 1, width]; 0: MLX [channels, width, 1]
    for (size_t fi = 0; fi < files.size(); ++fi) {
        std::map<std::string, Tensor> entries;
        rc = cp->parse_file(dir + "/" + files[fi], (int)fi, &entries);
        if (rc != QMR_OK) return rc;
        for (auto &kv : entries) {
            if (indexed) {
                auto it = weight_map.find(kv.first);
                if (it == weight_map.end() || it->second != files[fi])
                    return fail(QMR_EINVAL, "tensor %s missing or mapped to wrong shard", kv.first.c_str());
                seen.insert(kv.first);
            }
            Tensor t = kv.second;
            t.raw_hf = kv.first.rfind("model.language_model.", 0) == 0 ||
                       (kv.first.rfind("model.", 0) == 0 && !cp->has_default_quant_);
            const std::string canonical = canonical_name(kv.first);
            if (ends_with(canonical, ".linear_attn.conv1d.weight")) {
                const auto &s = t.shape;
                const uint32_t w = cp->cfg_.conv_width;
                if (s.size() != 3) return fail(QMR_EINVAL, "conv %s has invalid shape", canonical.c_str());
                const bool hf = s[1] == 1 && s[2] == w, mlx = s[1] == w && s[2] == 1;
                if (hf == mlx) return fail(QMR_EINVAL, "conv %s has ambiguous or invalid shape", canonical.c_str());
                const int layout = hf ? 1 : 0;
                if (conv_layout >= 0 && conv_layout != layout)
                    return fail(QMR_EINVAL, "checkpoint mixes HF and MLX conv layouts");
                conv_layout = layout;
            }
            if (!cp->tensors_.emplace(canonical, t).second)
                return fail(QMR_EINVAL, "duplicate canonical tensor %s", canonical.c_str());
        }
    }
    if (indexed && seen.size() != weight_map.size()) return fail(QMR_EINVAL, "index names missing from shards");
    // The conv orientation decides whether norms are zero-centred HF weights.
    if (conv_layout >= 0)
        for (auto &kv : cp->tensors_) kv.second.raw_hf = conv_layout == 1;
    *out = std::move(cp);
    return QMR_OK;
}

const Checkpoint::Tensor *Checkpoint::tensor(const std::string &key) const {
    auto it = tensors_.find(key);
    if (it != tensors_.end()) return &it->second;
    if (tied_ && key == "lm_head.weight") {
        auto e = tensors_.find("model.embed_tokens.weight");
        if (e != tensors_.end()) return &e->second;
    }
    return nullptr;
}

bool Checkpoint::contains(const std::string &name) const { return tensor(weight_key(name)) != nullptr; }

const uint8_t *Checkpoint::bytes(const Tensor &t) const {
    return static_cast<const uint8_t *>(files_[t.file].base) + t.offset;
}

int Checkpoint::floats(const Tensor &t, std::vector<float> *out) const {
    const uint8_t *p = bytes(t);
    if (t.dtype == "F32") {
        out->resize(t.length / 4);
        memcpy(out->data(), p, t.length);
    } else if (t.dtype == "F16") {
        out->resize(t.length / 2);
        for (size_t i = 0; i < out->size(); ++i) (*out)[i] = f16_to_f32(f16_bits_le(p + 2 * i));
    } else if (t.dtype == "BF16") {
        out->resize(t.length / 2);
        for (size_t i = 0; i < out->size(); ++i) {
            const uint32_t u = (uint32_t)f16_bits_le(p + 2 * i) << 16;
            memcpy(&(*out)[i], &u, 4);
        }
    } else {
        return fail(QMR_EINVAL, "tensor dtype %s is not floating point", t.dtype.c_str());
    }
    return QMR_OK;
}

int Checkpoint::matrix(const std::string &name, HostMatrix *m) const {
    const std::string key = weight_key(name);
    const Tensor *t = tensor(key);
    if (t == nullptr) return fail(QMR_EINVAL, "missing tensor %s", key.c_str());
    if (t->shape.size() != 2) return fail(QMR_EINVAL, "matrix %s must be rank 2", key.c_str());
    if (t->dtype != "U32") return fail(QMR_EUNSUPPORTED, "matrix %s is not packed (dense F16 weights are not on this path)", key.c_str());
    const std::string module = key.substr(0, key.size() - strlen(".weight"));
    QuantSpec q;
    bool have = has_default_quant_;
    q = default_quant_;
    auto ov = quant_overrides_.find(module);
    if (ov != quant_overrides_.end()) {
        have = ov->second.first;
        q = ov->second.second;
    }
    if (!have) return fail(QMR_EINVAL, "packed matrix %s lacks quantization metadata", key.c_str());
    const uint64_t words_per_group = q.group / (32 / q.bits);
    if (t->shape[1] % words_per_group != 0) return fail(QMR_EINVAL, "packed width not divisible by group width");
    const uint64_t groups = t->shape[1] / words_per_group;
    const uint64_t cols = groups * q.group;
    if (t->shape[0] > 0xffffffffull || cols > 0xffffffffull) return fail(QMR_ERANGE, "matrix %s too large", key.c_str());
    const uint64_t rows = t->shape[0];
    for (const char *part : {".scales", ".biases"}) {
        const Tensor *mt = tensor(module + part);
        if (mt == nullptr) return fail(QMR_EINVAL, "missing tensor %s%s", module.c_str(), part);
        if (mt->shape.size() != 2 || mt->shape[0] != rows || mt->shape[1] != groups)
            return fail(QMR_EINVAL, "%s%s shape mismatch", module.c_str(), part);
        std::vector<float> &dst = part[1] == 's' ? m->scales : m->biases;
        const int rc = floats(*mt, &dst);
        if (rc != QMR_OK) return rc;
        for (float v : dst)
            if (!std::isfinite(v)) return fail(QMR_EINVAL, "%s%s contains non-finite values", module.c_str(), part);
    }
    m->rows = (uint32_t)rows;
    m->cols = (uint32_t)cols;
    m->bits = q.bits;
    m->group = q.group;
    m->words.resize(t->length / 4);
    memcpy(m->words.data(), bytes(*t), t->length);  // little-endian u32, the host's order
    return QMR_OK;
}

int Checkpoint::vector(const std::string &name, std::vector<float> *v) const {
    const std::string key = weight_key(name);
    const Tensor *t = tensor(key);
    if (t == nullptr) return fail(QMR_EINVAL, "missing tensor %s", key.c_str());
    if (t->shape.size() != 1) return fail(QMR_EINVAL, "vector %s must be rank 1", key.c_str());
    int rc = floats(*t, v);
    if (rc != QMR_OK) return rc;
    if (t->raw_hf && zero_centered_norm(key))
        for (float &x : *v) x += 1.0f;
    for (float x : *v)
        if (!std::isfinite(x)) return fail(QMR_EINVAL, "vector %s has non-finite values", key.c_str());
    return QMR_OK;
}

int Checkpoint::conv(const std::string &name, uint32_t channels, uint32_t width, std::vector<float> *v) const {
    const std::string key = weight_key(name);
    const Tensor *t = tensor(key);
    if (t == nullptr) return fail(QMR_EINVAL, "missing tensor %s", key.c_str());
    const auto &s = t->shape;
    if (s.size() != 3 || s[0] != channels) return fail(QMR_EINVAL, "conv %s shape mismatch", key.c_str());
    if (!((s[1] == 1 && s[2] == width) || (s[1] == width && s[2] == 1)))
        return fail(QMR_EINVAL, "conv %s kernel shape mismatch", key.c_str());
    // Both layouts flatten to channel-major width.
    return floats(*t, v);
}

}  // namespace qmr
