// Model runtime of liblsx: checkpoint loading and the Model API of the reference
// (src/model.rs:383-853), executed either by the fused decode engine (decode.cu)
// or, for checkpoints outside its envelope (F32/F16 projections, LayerNorm,
// odd head sizes), by the per-op kernels in the exact op order of
// Model::decode.  Both plans run on the GPU; there is no host compute path.
#include <dirent.h>
#include <stdio.h>
#include <stdlib.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <fstream>
#include <memory>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "batched.cuh"
#include "decode.cuh"
#include "persistent.cuh"
#include "device_common.cuh"
#include "json.h"
#include "lsx_internal.h"

namespace lsx {

// ------------------------------------------------------------ checkpoint --
struct Mapped {
    void* base = nullptr;
    size_t size = 0;
    ~Mapped() {
        if (base) munmap(base, size);
    }
};

struct Entry {
    size_t file = 0;
    std::string dtype;
    std::vector<size_t> shape;
    const unsigned char* data = nullptr;
    size_t bytes = 0;
    size_t count() const {
        size_t n = 1;
        for (size_t d : shape) n *= d;
        return n;
    }
};

struct Checkpoint {
    std::vector<std::unique_ptr<Mapped>> files;
    std::map<std::string, Entry> entries;
};

static std::string read_text(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

static bool is_file(const std::string& path) {
    struct stat st;
    return stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

static bool ends_with(const std::string& s, const std::string& suffix) {
    return s.size() >= suffix.size() && s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0;
}

// hub::weight_files (src/hub.rs:67-128)
static std::vector<std::string> weight_files(const std::string& root) {
    std::set<std::string> names;
    DIR* d = opendir(root.c_str());
    if (!d) throw std::runtime_error("cannot open model folder " + root);
    while (dirent* e = readdir(d)) names.insert(e->d_name);
    closedir(d);
    std::string index;
    if (names.count("model.safetensors.index.json")) {
        index = "model.safetensors.index.json";
    } else {
        int found = 0;
        for (auto& n : names)
            if (ends_with(n, ".safetensors.index.json")) {
                index = n;
                ++found;
            }
        if (found > 1) throw std::runtime_error("the model folder must hold one weight index");
    }
    std::set<std::string> chosen;
    if (!index.empty()) {
        json::Value v = json::parse(read_text(root + "/" + index));
        const json::Value& map = v["weight_map"];
        if (!map.is_object()) throw std::runtime_error("weight index has no weight_map");
        for (auto& m : map.members) {
            if (!m.second.is_string() || !ends_with(m.second.text, ".safetensors") ||
                m.second.text.find("..") != std::string::npos || m.second.text[0] == '/')
                throw std::runtime_error("weight shards must be relative safetensors names");
            chosen.insert(m.second.text);
        }
    } else if (names.count("model.safetensors")) {
        chosen.insert("model.safetensors");
    } else {
        for (auto& n : names)
            if (ends_with(n, ".safetensors") && n != "adapter_model.safetensors") chosen.insert(n);
        if (chosen.size() != 1) throw std::runtime_error("choose a single weight file or a shard index");
    }
    return std::vector<std::string>(chosen.begin(), chosen.end());
}

// Checkpoint::open (src/model.rs:59-91)
static void open_checkpoint(const std::string& root, Checkpoint& ck) {
    auto names = weight_files(root);
    if (names.empty()) throw std::runtime_error("safetensors model weights are required");
    for (auto& name : names) {
        std::string path = root + "/" + name;
        int fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) throw std::runtime_error("cannot open " + path);
        struct stat st;
        fstat(fd, &st);
        auto m = std::make_unique<Mapped>();
        m->size = (size_t)st.st_size;
        m->base = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (m->base == MAP_FAILED) {
            m->base = nullptr;
            throw std::runtime_error("cannot map " + path);
        }
        if (m->size < 8) throw std::runtime_error(name + ": truncated safetensors file");
        uint64_t header = 0;
        memcpy(&header, m->base, 8);
        if (header > m->size - 8) throw std::runtime_error(name + ": bad safetensors header length");
        const char* h = (const char*)m->base + 8;
        json::Value meta = json::Parser(h, (size_t)header).parse();
        const unsigned char* data = (const unsigned char*)m->base + 8 + header;
        size_t data_size = m->size - 8 - header;
        for (auto& kv : meta.members) {
            if (kv.first == "__metadata__") continue;
            Entry e;
            e.file = ck.files.size();
            e.dtype = kv.second["dtype"].text;
            for (auto& d : kv.second["shape"].items) e.shape.push_back((size_t)d.u64());
            const json::Value& off = kv.second["data_offsets"];
            if (!off.is_array() || off.items.size() != 2) throw std::runtime_error(kv.first + ": data_offsets");
            size_t b = (size_t)off.items[0].u64(), en = (size_t)off.items[1].u64();
            if (b > en || en > data_size) throw std::runtime_error(kv.first + ": data outside the file");
            e.data = data + b;
            e.bytes = en - b;
            if (ck.entries.count(kv.first)) throw std::runtime_error("duplicate weight name: " + kv.first);
            ck.entries[kv.first] = e;
        }
        ck.files.push_back(std::move(m));
    }
}

static int dtype_code(const std::string& d) {
    if (d == "F32") return LSX_F32;
    if (d == "F16") return LSX_F16;
    if (d == "BF16") return LSX_BF16;
    return -1;
}

static float bf16_bits_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else {
            int e = -1;
            do {
                man <<= 1;
                ++e;
            } while (!(man & 0x400u));
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// Checkpoint::floats (src/model.rs:115-135)
static std::vector<float> floats(const Entry& e) {
    std::vector<float> out(e.count());
    int k = dtype_code(e.dtype);
    for (size_t i = 0; i < out.size(); ++i) {
        if (k == LSX_F32) memcpy(&out[i], e.data + 4 * i, 4);
        else {
            uint16_t b;
            memcpy(&b, e.data + 2 * i, 2);
            out[i] = k == LSX_BF16 ? bf16_bits_to_f32(b) : f16_bits_to_f32(b);
        }
    }
    return out;
}

// -------------------------------------------------------------- graph spec --
struct NormSpec {
    std::string weight, bias;
    bool layer = false;
    float epsilon = 0.f;
    float gain_offset = 0.f;
};
struct LinearSpec {
    std::string weight, bias;
};
struct BlockSpec {
    NormSpec input, post;
    LinearSpec q, k, v, o, gate, up, down;
    bool has_qn = false, has_kn = false;
    NormSpec qn, kn;
    size_t qheads = 0, kvheads = 0, head_dim = 0, rotary = 0, intermediate = 0;
    float theta = 0.f, scale = 0.f;
    bool interleaved = false;
    int activation = 0;
};
struct GraphSpec {
    size_t hidden = 0, vocab = 0, max_context = 0;
    std::string embedding;
    float embedding_scale = 1.f;
    NormSpec final_norm;
    LinearSpec readout;
    std::vector<BlockSpec> blocks;
    std::vector<uint32_t> eos;
};

static size_t req(const json::Value& c, const char* key) {
    const json::Value& v = c[key];
    if (!v.is_integer() || v.text[0] == '-') throw std::runtime_error(std::string("config integer ") + key);
    return (size_t)v.u64();
}

static int activation_code(const std::string& name) {
    if (name == "silu" || name == "swish") return 0;
    if (name == "gelu") return 1;
    if (name == "relu") return 2;
    if (name == "gelu_new" || name == "gelu_fast" || name == "gelu_pytorch_tanh" || name == "gelu_tanh") return 3;
    throw std::runtime_error("activation " + name + " needs its operation defined");
}

// GraphSpec::from_config (src/graph.rs:231-411)
static GraphSpec from_config(const json::Value& c, const Checkpoint& ck) {
    std::vector<std::string> prefixes;
    const std::string suffix = ".0.self_attn.q_proj.weight";
    for (auto& kv : ck.entries)
        if (ends_with(kv.first, suffix)) prefixes.push_back(kv.first.substr(0, kv.first.size() - suffix.size()));
    if (prefixes.size() != 1)
        throw std::runtime_error("a single decoder with separate Q/K/V weights, or laplace.graph.json, is required");
    std::string prefix = prefixes[0], stem;
    if (ends_with(prefix, ".layers")) stem = prefix.substr(0, prefix.size() - 7) + ".";
    else if (prefix == "layers") stem = "";
    else throw std::runtime_error("decoder layers path");
    auto has = [&](const std::string& n) { return ck.entries.count(n) > 0; };
    auto linear = [&](const std::string& name) {
        LinearSpec l;
        l.weight = name + ".weight";
        if (has(name + ".bias")) l.bias = name + ".bias";
        return l;
    };
    if (!c["rms_norm_eps"].is_number()) throw std::runtime_error("config rms_norm_eps");
    const float epsilon = (float)c["rms_norm_eps"].number();
    const bool gemma = c["model_type"].is_string() && c["model_type"].text == "gemma";
    const float offset = gemma ? 1.f : 0.f;
    auto rms = [&](const std::string& name, float off) {
        NormSpec n;
        n.weight = name + ".weight";
        n.epsilon = epsilon;
        n.gain_offset = off;
        return n;
    };
    GraphSpec g;
    g.hidden = req(c, "hidden_size");
    size_t heads = req(c, "num_attention_heads");
    size_t kv = c["num_key_value_heads"].is_null() ? heads : req(c, "num_key_value_heads");
    size_t dim = c["head_dim"].is_null() ? (heads ? g.hidden / heads : 0) : req(c, "head_dim");
    double ratio = c["partial_rotary_factor"].is_null() ? 1.0 : c["partial_rotary_factor"].number();
    double rotary = (double)dim * ratio;
    if (!std::isfinite(ratio) || ratio < 0 || ratio > 1 || std::fabs(rotary - std::floor(rotary)) > 1e-8)
        throw std::runtime_error("partial_rotary_factor must give an integer rotary dimension");
    for (const char* key : {"rope_scaling", "attn_logit_softcapping", "final_logit_softcapping", "num_local_experts",
                            "num_experts"})
        if (!c[key].is_null()) throw std::runtime_error(std::string("config ") + key + " needs an extended operation");
    bool sliding = c["use_sliding_window"].is_bool() && c["use_sliding_window"].boolean;
    bool window_off = c["use_sliding_window"].is_bool() && !c["use_sliding_window"].boolean;
    if (sliding || !(c["sliding_window"].is_null() || window_off))
        throw std::runtime_error("sliding window attention needs an extended attention op");
    const json::Value& rp = c["rope_parameters"];
    if (rp["rope_type"].is_string() && rp["rope_type"].text != "default")
        throw std::runtime_error("the configured RoPE type needs its frequency op");
    double theta;
    if (c["rope_theta"].is_number()) theta = c["rope_theta"].number();
    else if (rp["rope_theta"].is_number()) theta = rp["rope_theta"].number();
    else throw std::runtime_error("config rope_theta");
    std::string act = "silu";
    if (c["hidden_activation"].is_string()) act = c["hidden_activation"].text;
    else if (c["hidden_act"].is_string()) act = c["hidden_act"].text;
    int activation = activation_code(act);
    bool interleaved = false;
    if (c["rope_interleaved"].is_bool()) interleaved = c["rope_interleaved"].boolean;
    else if (c["rotary_interleaved"].is_bool()) interleaved = c["rotary_interleaved"].boolean;
    size_t layers = req(c, "num_hidden_layers");
    size_t inter = req(c, "intermediate_size");
    for (size_t i = 0; i < layers; ++i) {
        std::string layer = prefix + "." + std::to_string(i);
        std::string attn = layer + ".self_attn";
        if (has(layer + ".pre_feedforward_layernorm.weight") || has(layer + ".post_feedforward_layernorm.weight"))
            throw std::runtime_error("extra residual norms need an explicit execution graph");
        BlockSpec b;
        b.input = rms(layer + ".input_layernorm", offset);
        b.post = rms(layer + ".post_attention_layernorm", offset);
        b.q = linear(attn + ".q_proj");
        b.k = linear(attn + ".k_proj");
        b.v = linear(attn + ".v_proj");
        b.o = linear(attn + ".o_proj");
        if (has(attn + ".q_norm.weight")) {
            b.has_qn = true;
            b.qn = rms(attn + ".q_norm", 0.f);
        }
        if (has(attn + ".k_norm.weight")) {
            b.has_kn = true;
            b.kn = rms(attn + ".k_norm", 0.f);
        }
        b.qheads = heads;
        b.kvheads = kv;
        b.head_dim = dim;
        b.rotary = (size_t)rotary;
        b.theta = (float)theta;
        b.interleaved = interleaved;
        b.scale = 1.f / std::sqrt((float)dim);
        b.gate = linear(layer + ".mlp.gate_proj");
        b.up = linear(layer + ".mlp.up_proj");
        b.down = linear(layer + ".mlp.down_proj");
        b.intermediate = inter;
        b.activation = activation;
        g.blocks.push_back(b);
    }
    g.embedding = stem + "embed_tokens.weight";
    if (c["tie_word_embeddings"].is_bool() && c["tie_word_embeddings"].boolean) {
        g.readout.weight = g.embedding;
        if (has("lm_head.bias")) g.readout.bias = "lm_head.bias";
    } else {
        g.readout = linear("lm_head");
    }
    const json::Value& eos = c["eos_token_id"];
    if (eos.is_array()) {
        for (auto& v : eos.items) {
            if (!v.is_integer()) throw std::runtime_error("EOS integer id");
            g.eos.push_back((uint32_t)v.u64());
        }
    } else if (!eos.is_null()) {
        if (!eos.is_integer()) throw std::runtime_error("EOS integer id");
        g.eos.push_back((uint32_t)eos.u64());
    }
    g.vocab = req(c, "vocab_size");
    g.max_context = req(c, "max_position_embeddings");
    g.embedding_scale = gemma ? std::sqrt((float)g.hidden) : 1.f;
    g.final_norm = rms(stem + "norm", offset);
    return g;
}

static NormSpec norm_from_json(const json::Value& v) {
    NormSpec n;
    n.weight = v["weight"].text;
    if (v["bias"].is_string()) n.bias = v["bias"].text;
    if (!v["kind"].is_string()) throw std::runtime_error("norm kind");
    if (v["kind"].text == "layer") n.layer = true;
    else if (v["kind"].text != "rms") throw std::runtime_error("norm kind must be rms or layer");
    n.epsilon = (float)v["epsilon"].number();
    if (v["gain_offset"].is_number()) n.gain_offset = (float)v["gain_offset"].number();
    return n;
}
static LinearSpec linear_from_json(const json::Value& v) {
    LinearSpec l;
    if (!v["weight"].is_string()) throw std::runtime_error("linear weight name");
    l.weight = v["weight"].text;
    if (v["bias"].is_string()) l.bias = v["bias"].text;
    return l;
}

// Deserialising laplace.graph.json (src/graph.rs:93-107)
static GraphSpec from_graph_json(const json::Value& v) {
    if (!v["version"].is_integer() || v["version"].u64() != 1)
        throw std::runtime_error("the execution graph must be version 1");
    GraphSpec g;
    g.hidden = req(v, "hidden_size");
    g.vocab = req(v, "vocab_size");
    g.max_context = req(v, "max_context");
    g.embedding = v["embedding"].text;
    if (v["embedding_scale"].is_number()) g.embedding_scale = (float)v["embedding_scale"].number();
    g.final_norm = norm_from_json(v["final_norm"]);
    g.readout = linear_from_json(v["readout"]);
    for (auto& b : v["blocks"].items) {
        BlockSpec s;
        s.input = norm_from_json(b["input_norm"]);
        s.post = norm_from_json(b["post_attention_norm"]);
        const json::Value& a = b["attention"];
        s.q = linear_from_json(a["query"]);
        s.k = linear_from_json(a["key"]);
        s.v = linear_from_json(a["value"]);
        s.o = linear_from_json(a["output"]);
        if (a["query_norm"].is_object()) {
            s.has_qn = true;
            s.qn = norm_from_json(a["query_norm"]);
        }
        if (a["key_norm"].is_object()) {
            s.has_kn = true;
            s.kn = norm_from_json(a["key_norm"]);
        }
        s.qheads = req(a, "query_heads");
        s.kvheads = req(a, "kv_heads");
        s.head_dim = req(a, "head_dim");
        s.rotary = req(a, "rotary_dim");
        s.theta = (float)a["rope_theta"].number();
        if (a["rotary_interleaved"].is_bool()) s.interleaved = a["rotary_interleaved"].boolean;
        s.scale = (float)a["score_scale"].number();
        const json::Value& m = b["mlp"];
        s.gate = linear_from_json(m["gate"]);
        s.up = linear_from_json(m["up"]);
        s.down = linear_from_json(m["down"]);
        s.intermediate = req(m, "intermediate_size");
        s.activation = activation_code(m["activation"].text);
        g.blocks.push_back(s);
    }
    for (auto& e : v["eos_token_ids"].items) g.eos.push_back((uint32_t)e.u64());
    return g;
}

// GraphSpec::validate with its Contract (src/graph.rs:108-229)
static void validate(const GraphSpec& g, const Checkpoint& ck) {
    if (!(g.hidden > 0 && g.vocab > 1 && g.vocab <= 0xffffffffull && g.max_context > 0 && !g.blocks.empty()))
        throw std::runtime_error("check the decoder dimensions and block count");
    if (!std::isfinite(g.embedding_scale)) throw std::runtime_error("embedding scale must be finite");
    for (uint32_t t : g.eos)
        if (t >= g.vocab) throw std::runtime_error("EOS token outside the vocabulary");
    auto tensor = [&](const std::string& name, std::vector<size_t> dims) {
        auto it = ck.entries.find(name);
        if (it == ck.entries.end()) throw std::runtime_error("tensor required by the graph: " + name);
        if (it->second.shape != dims) throw std::runtime_error(name + ": stored shape does not match");
        if (dtype_code(it->second.dtype) < 0) throw std::runtime_error(name + ": store F32/F16/BF16");
        size_t count = it->second.count();
        if (count == 0 || count > 2147483647ull) throw std::runtime_error(name + ": index range must be 1..=i32::MAX");
        if (it->second.bytes != count * dtype_bytes(dtype_code(it->second.dtype)))
            throw std::runtime_error(name + ": byte size does not match its shape");
    };
    auto linear = [&](const LinearSpec& p, size_t in, size_t out) {
        tensor(p.weight, {out, in});
        if (!p.bias.empty()) tensor(p.bias, {out});
    };
    auto norm = [&](const NormSpec& n, size_t width) {
        if (!(std::isfinite(n.epsilon) && n.epsilon > 0 && std::isfinite(n.gain_offset)))
            throw std::runtime_error("norm epsilon must be positive and gain offset finite");
        tensor(n.weight, {width});
        if (!n.bias.empty()) tensor(n.bias, {width});
    };
    tensor(g.embedding, {g.vocab, g.hidden});
    norm(g.final_norm, g.hidden);
    linear(g.readout, g.hidden, g.vocab);
    for (auto& b : g.blocks) {
        norm(b.input, g.hidden);
        norm(b.post, g.hidden);
        if (!(b.qheads > 0 && b.kvheads > 0 && b.head_dim > 0 && b.qheads % b.kvheads == 0))
            throw std::runtime_error("query heads must be a positive multiple of KV heads");
        if (!(b.rotary <= b.head_dim && b.rotary % 2 == 0))
            throw std::runtime_error("rotary dim must be even and at most head_dim");
        if (!(std::isfinite(b.theta) && b.theta > 0 && std::isfinite(b.scale) && b.scale > 0))
            throw std::runtime_error("RoPE base and attention scale must be positive");
        size_t q = b.qheads * b.head_dim, kv = b.kvheads * b.head_dim;
        linear(b.q, g.hidden, q);
        linear(b.k, g.hidden, kv);
        linear(b.v, g.hidden, kv);
        linear(b.o, q, g.hidden);
        if (b.has_qn) norm(b.qn, b.head_dim);
        if (b.has_kn) norm(b.kn, b.head_dim);
        if (b.intermediate == 0) throw std::runtime_error("MLP width must be positive");
        linear(b.gate, g.hidden, b.intermediate);
        linear(b.up, g.hidden, b.intermediate);
        linear(b.down, b.intermediate, g.hidden);
    }
}

// argmax over a device vector: first maximum, as src/diagnosis.rs:58-70.
__global__ void argmax_kernel(const float* z, int n, unsigned long long* out, int* nonfinite) {
    unsigned long long best = 0ull;
    bool bad = false;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float v = z[i];
        bad |= !isfinite(v);
        unsigned long long k = pack_arg(v, (uint32_t)i);
        best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) atomicMax(out, best);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(nonfinite, 1);
}

// Teacher-forced loss of one scored position per block: attribution::loss
// (src/attribution.rs:49-60), top + ln(sum_j exp(z_j - top)) - z[target], in f64.
__global__ void __launch_bounds__(1024) frame_nll_kernel(const float* __restrict__ logits, int vocab,
                                                         const uint32_t* __restrict__ targets, double* nll) {
    __shared__ double red[32];
    const float* z = logits + (size_t)blockIdx.x * vocab;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double top = -INFINITY;
    for (int j = tid; j < vocab; j += blockDim.x) top = fmax(top, (double)z[j]);
    for (int o = 16; o > 0; o >>= 1) top = fmax(top, __shfl_xor_sync(0xffffffffu, top, o));
    if (lane == 0) red[warp] = top;
    __syncthreads();
    top = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) top = fmax(top, red[w]);
    __syncthreads();
    double sum = 0.0;
    for (int j = tid; j < vocab; j += blockDim.x) sum += exp((double)z[j] - top);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        double total = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total += red[w];
        nll[blockIdx.x] = top + log(total) - (double)z[targets[blockIdx.x]];
    }
}

}  // namespace lsx

using namespace lsx;

// ------------------------------------------------------------------- model --
struct lsx_model {
    lsx_ctx* ctx = nullptr;
    GraphSpec graph;
    size_t capacity = 0, cursor = 0;
    uint64_t parameters = 0, tensors = 0;
    std::map<std::string, lsx_tensor*> bank;  // Bank (src/model.rs:137-152), stored kinds
    std::vector<lsx_tensor*> owned;
    struct Norm {
        lsx_tensor* gain = nullptr;
        lsx_tensor* bias = nullptr;
        size_t groups = 1, width = 0;
        float eps = 0.f;
        bool center = false;
    };
    struct Proj {
        lsx_tensor* weight = nullptr;
        lsx_tensor* bias = nullptr;  // f32
        size_t in = 0, out = 0;
    };
    struct Block {
        Norm input, post, qn, kn;
        bool has_qn = false, has_kn = false;
        Proj q, k, v, o, gate, up, down;
        lsx_tensor* keys = nullptr;
        lsx_tensor* values = nullptr;
    };
    std::vector<Block> blocks;
    Norm final_norm;
    Proj head;
    lsx_tensor* embedding = nullptr;
    bool fused = false;
    std::unique_ptr<FusedDecoder> decoder;
    std::unique_ptr<PersistentDecoder> persistent;  // preferred fused engine when it fits
    std::unique_ptr<BatchedScorer> batched;          // batched teacher forcing (built on first use)
    FusedConfig fused_config{};
    std::vector<FusedLayer> fused_layers;
    unsigned int epoch = 0;                           // tagged-buffer epoch of the persistent engine
    // Per-op plan work buffers.
    std::vector<lsx_tensor*> work;
    // Host<->device staging for the fused plan.
    DecodeState* host_state = nullptr;  // pinned
    uint32_t* d_prompt = nullptr;
    uint32_t* d_tokens = nullptr;
    float* d_inject = nullptr;
    float* d_hidden1 = nullptr;
    float* d_logits1 = nullptr;
    float* d_frames = nullptr;
    size_t frames_capacity = 0;  // in tokens
    unsigned long long* d_best = nullptr;
    int* d_flag = nullptr;
    ~lsx_model();
};

lsx_model::~lsx_model() {
    if (ctx) {
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
    }
    decoder.reset();
    persistent.reset();
    batched.reset();
    for (auto& kv : bank) lsx_tensor_free(kv.second);
    for (auto* t : owned) lsx_tensor_free(t);
    for (auto* t : work) lsx_tensor_free(t);
    for (void* p : {(void*)d_prompt, (void*)d_tokens, (void*)d_inject, (void*)d_hidden1, (void*)d_logits1,
                    (void*)d_frames, (void*)d_best, (void*)d_flag})
        if (p) cudaFree(p);
    if (host_state) cudaFreeHost(host_state);
}

namespace {

int upload_entry(lsx_ctx* ctx, const Entry& e, lsx_tensor** out) {
    return lsx_upload_raw(ctx, e.data, e.bytes, (lsx_dtype)dtype_code(e.dtype), out);
}

int bank_take(lsx_model* m, const Checkpoint& ck, const std::string& name, lsx_tensor** out) {
    auto it = m->bank.find(name);
    if (it != m->bank.end()) {
        *out = it->second;
        return LSX_OK;
    }
    lsx_tensor* t = nullptr;
    LSX_TRY(upload_entry(m->ctx, ck.entries.at(name), &t));
    m->bank[name] = t;
    *out = t;
    return LSX_OK;
}

int upload_f32_vec(lsx_model* m, const std::vector<float>& v, lsx_tensor** out) {
    LSX_TRY(lsx_upload_f32(m->ctx, v.data(), v.size(), out));
    m->owned.push_back(*out);
    return LSX_OK;
}

// Normalization::bind (src/model.rs:224-253): gains widened to f32 plus gain_offset.
int bind_norm(lsx_model* m, const Checkpoint& ck, const NormSpec& s, size_t groups, size_t width,
              lsx_model::Norm* n) {
    std::vector<float> g = floats(ck.entries.at(s.weight));
    for (float& x : g) {
        x += s.gain_offset;
        if (!std::isfinite(x)) return fail(LSX_E_FORMAT, "norm gains must be finite");
    }
    LSX_TRY(upload_f32_vec(m, g, &n->gain));
    if (!s.bias.empty()) LSX_TRY(upload_f32_vec(m, floats(ck.entries.at(s.bias)), &n->bias));
    n->groups = groups;
    n->width = width;
    n->eps = s.epsilon;
    n->center = s.layer;
    return LSX_OK;
}

int bind_proj(lsx_model* m, const Checkpoint& ck, const LinearSpec& s, size_t in, size_t out, bool upload,
              lsx_model::Proj* p) {
    if (upload) LSX_TRY(bank_take(m, ck, s.weight, &p->weight));
    if (!s.bias.empty()) LSX_TRY(upload_f32_vec(m, floats(ck.entries.at(s.bias)), &p->bias));
    p->in = in;
    p->out = out;
    return LSX_OK;
}

int work_buffer(lsx_model* m, size_t count, float** out) {
    lsx_tensor* t = nullptr;
    LSX_TRY(reserve(m->ctx, count, LSX_F32, &t));
    m->work.push_back(t);
    *out = (float*)t->data;
    return LSX_OK;
}

bool fusable(const GraphSpec& g, const Checkpoint& ck) {
    const BlockSpec& b0 = g.blocks[0];
    for (auto& b : g.blocks) {
        if (b.qheads != b0.qheads || b.kvheads != b0.kvheads || b.head_dim != b0.head_dim || b.rotary != b0.rotary ||
            b.intermediate != b0.intermediate || b.activation != b0.activation || b.theta != b0.theta ||
            b.interleaved != b0.interleaved || b.scale != b0.scale)
            return false;
        if (b.input.layer || b.post.layer || !b.input.bias.empty() || !b.post.bias.empty()) return false;
        if (b.input.epsilon != g.blocks[0].input.epsilon || b.post.epsilon != g.blocks[0].input.epsilon) return false;
        if (b.has_qn != b0.has_qn || b.has_kn != b0.has_kn) return false;
        if ((b.has_qn && (b.qn.layer || !b.qn.bias.empty())) || (b.has_kn && (b.kn.layer || !b.kn.bias.empty())))
            return false;
        if (b.has_qn && b.has_kn && b.qn.epsilon != b.kn.epsilon) return false;
        for (const LinearSpec* p : {&b.q, &b.k, &b.v, &b.o, &b.gate, &b.up, &b.down})
            if (ck.entries.at(p->weight).dtype != "BF16") return false;
    }
    if (g.final_norm.layer || !g.final_norm.bias.empty() || g.final_norm.epsilon != g.blocks[0].input.epsilon)
        return false;
    if (ck.entries.at(g.readout.weight).dtype != "BF16") return false;
    return true;
}

// Copies rows into one device buffer, interleaving or concatenating.
int upload_rows(lsx_model* m, const std::vector<std::pair<const Entry*, size_t>>& pieces, size_t row_bytes,
                bool interleave, lsx_tensor** out) {
    size_t rows = 0;
    for (auto& p : pieces) rows += p.second;
    std::vector<unsigned char> host(rows * row_bytes);
    if (interleave) {  // pieces[0], pieces[1] have equal row counts: row 2f = a_f, 2f+1 = b_f
        size_t n = pieces[0].second;
        for (size_t f = 0; f < n; ++f) {
            memcpy(&host[(2 * f) * row_bytes], pieces[0].first->data + f * row_bytes, row_bytes);
            memcpy(&host[(2 * f + 1) * row_bytes], pieces[1].first->data + f * row_bytes, row_bytes);
        }
    } else {
        size_t at = 0;
        for (auto& p : pieces) {
            memcpy(&host[at], p.first->data, p.second * row_bytes);
            at += p.second * row_bytes;
        }
    }
    LSX_TRY(lsx_upload_raw(m->ctx, host.data(), host.size(), LSX_BF16, out));
    m->owned.push_back(*out);
    return LSX_OK;
}

int concat_bias(lsx_model* m, const Checkpoint& ck, const std::vector<std::pair<std::string, size_t>>& parts,
                bool interleave, lsx_tensor** out) {
    bool any = false;
    for (auto& p : parts) any |= !p.first.empty();
    *out = nullptr;
    if (!any) return LSX_OK;
    std::vector<std::vector<float>> vals;
    for (auto& p : parts) vals.push_back(p.first.empty() ? std::vector<float>(p.second, 0.f)
                                                        : floats(ck.entries.at(p.first)));
    std::vector<float> all;
    if (interleave) {
        for (size_t f = 0; f < parts[0].second; ++f) {
            all.push_back(vals[0][f]);
            all.push_back(vals[1][f]);
        }
    } else {
        for (auto& v : vals) all.insert(all.end(), v.begin(), v.end());
    }
    return upload_f32_vec(m, all, out);
}

// ---------------------------------------------------------- per-op plan ----
struct OpBuffers {
    float *residual, *norm, *q, *k, *v, *t, *mixed, *proj, *gate, *up, *feature, *hidden, *rotated, *logits;
};

int op_buffers(lsx_model* m, OpBuffers* b) {
    const GraphSpec& g = m->graph;
    size_t qw = 0, kw = 0, I = 0;
    for (auto& s : g.blocks) {
        qw = std::max(qw, s.qheads * s.head_dim);
        kw = std::max(kw, s.kvheads * s.head_dim);
        I = std::max(I, s.intermediate);
    }
    size_t big = std::max({qw, g.hidden, I});
    LSX_TRY(work_buffer(m, g.hidden, &b->residual));
    LSX_TRY(work_buffer(m, big, &b->norm));
    LSX_TRY(work_buffer(m, qw, &b->q));
    LSX_TRY(work_buffer(m, kw, &b->k));
    LSX_TRY(work_buffer(m, kw, &b->v));
    LSX_TRY(work_buffer(m, big, &b->t));
    LSX_TRY(work_buffer(m, qw, &b->mixed));
    LSX_TRY(work_buffer(m, g.hidden, &b->proj));
    LSX_TRY(work_buffer(m, I, &b->gate));
    LSX_TRY(work_buffer(m, I, &b->up));
    LSX_TRY(work_buffer(m, I, &b->feature));
    LSX_TRY(work_buffer(m, g.hidden, &b->hidden));
    LSX_TRY(work_buffer(m, g.hidden, &b->rotated));
    LSX_TRY(work_buffer(m, g.vocab, &b->logits));
    return LSX_OK;
}

OpBuffers buffers_of(lsx_model* m) {
    OpBuffers b;
    float** f = (float**)&b;
    for (size_t i = 0; i < sizeof(OpBuffers) / sizeof(float*); ++i) f[i] = (float*)m->work[i]->data;
    return b;
}

#define LSX_K(call, what)                                                     \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess) return fail(LSX_E_CUDA, cuda_message(what, e_)); \
    } while (0)

int run_norm(lsx_model* m, const lsx_model::Norm& n, const float* x, float* out) {
    LSX_K(launch_norm(m->ctx->stream, x, (const float*)n.gain->data, n.bias ? (const float*)n.bias->data : nullptr,
                      n.groups, n.width, n.eps, n.center, out),
          "normalization");
    return LSX_OK;
}
int run_proj(lsx_model* m, const lsx_model::Proj& p, const float* x, float* out, bool with_bias = true) {
    LSX_K(launch_matvec(m->ctx->stream, m->ctx->sm_count, p.weight->data, p.weight->kind, x,
                        (with_bias && p.bias) ? (const float*)p.bias->data : nullptr, p.out, p.in, out,
                        true),  // checkpoint weights: uploaded once, never written
          "matvec");
    return LSX_OK;
}

// Rotation application on device buffers (DeviceRotation::apply, src/model.rs:342-363).
int apply_rotation(lsx_ctx* ctx, const lsx_rotation* r, const float* h, float* out, float* t1, float* t2, float* t3) {
    cudaStream_t s = ctx->stream;
    if (!r->joint) {
        LSX_K(launch_rotate(s, h, (const float*)r->u->data, (const float*)r->v->data, r->cosine_minus_one, r->sine,
                            r->width, out),
              "plane_rotation");
        return LSX_OK;
    }
    LSX_K(launch_matvec(s, ctx->sm_count, r->basis->data, LSX_F32, h, nullptr, r->rank, r->width, t1), "matvec");
    LSX_K(launch_matvec(s, ctx->sm_count, r->delta->data, LSX_F32, t1, nullptr, r->rank, r->rank, t2), "matvec");
    LSX_K(launch_matvec(s, ctx->sm_count, r->transpose->data, LSX_F32, t2, nullptr, r->width, r->rank, t3), "matvec");
    LSX_K(launch_combine(s, h, t3, 1.f, r->width, out), "vector_sum");
    return LSX_OK;
}

// Model::decode (src/model.rs:729-853) with per-op kernels on device buffers.
int decode_ops(lsx_model* m, const lsx_rotation* rotation, float** logits_out) {
    const GraphSpec& g = m->graph;
    OpBuffers b = buffers_of(m);
    cudaStream_t s = m->ctx->stream;
    const size_t pos = m->cursor;
    for (size_t l = 0; l < m->blocks.size(); ++l) {
        const lsx_model::Block& B = m->blocks[l];
        const BlockSpec& S = g.blocks[l];
        size_t qw = S.qheads * S.head_dim, kw = S.kvheads * S.head_dim;
        LSX_TRY(run_norm(m, B.input, b.residual, b.norm));
        LSX_TRY(run_proj(m, B.q, b.norm, b.q));
        LSX_TRY(run_proj(m, B.k, b.norm, b.k));
        LSX_TRY(run_proj(m, B.v, b.norm, b.v));
        if (B.has_qn) {
            LSX_TRY(run_norm(m, B.qn, b.q, b.t));
            LSX_K(cudaMemcpyAsync(b.q, b.t, qw * 4, cudaMemcpyDeviceToDevice, s), "copy");
        }
        if (B.has_kn) {
            LSX_TRY(run_norm(m, B.kn, b.k, b.t));
            LSX_K(cudaMemcpyAsync(b.k, b.t, kw * 4, cudaMemcpyDeviceToDevice, s), "copy");
        }
        if (S.rotary > 0) {
            LSX_K(launch_rope(s, b.q, pos, S.qheads, S.head_dim, S.theta, S.rotary, S.interleaved, b.t), "rope");
            LSX_K(cudaMemcpyAsync(b.q, b.t, qw * 4, cudaMemcpyDeviceToDevice, s), "copy");
            LSX_K(launch_rope(s, b.k, pos, S.kvheads, S.head_dim, S.theta, S.rotary, S.interleaved, b.t), "rope");
            LSX_K(cudaMemcpyAsync(b.k, b.t, kw * 4, cudaMemcpyDeviceToDevice, s), "copy");
        }
        LSX_K(launch_cache_write(s, b.k, b.v, (float*)B.keys->data, (float*)B.values->data, pos, kw), "cache_write");
        LSX_K(launch_attention(s, b.q, (const float*)B.keys->data, (const float*)B.values->data, pos, S.qheads,
                               S.kvheads, S.head_dim, S.scale, b.mixed),
              "causal_attention");
        LSX_TRY(run_proj(m, B.o, b.mixed, b.proj));
        LSX_K(launch_combine(s, b.residual, b.proj, 1.f, g.hidden, b.residual), "vector_sum");
        LSX_TRY(run_norm(m, B.post, b.residual, b.norm));
        LSX_TRY(run_proj(m, B.gate, b.norm, b.gate));
        LSX_TRY(run_proj(m, B.up, b.norm, b.up));
        LSX_K(launch_gated(s, b.gate, b.up, S.intermediate, S.activation, b.feature), "gated_product");
        LSX_TRY(run_proj(m, B.down, b.feature, b.proj));
        LSX_K(launch_combine(s, b.residual, b.proj, 1.f, g.hidden, b.residual), "vector_sum");
    }
    LSX_TRY(run_norm(m, m->final_norm, b.residual, b.hidden));
    const float* input = b.hidden;
    if (rotation) {
        LSX_TRY(apply_rotation(m->ctx, rotation, b.hidden, b.rotated, b.norm, b.t, b.proj));
        input = b.rotated;
    }
    LSX_TRY(run_proj(m, m->head, input, b.logits));
    *logits_out = b.logits;
    return LSX_OK;
}

int embedding_into(lsx_model* m, uint32_t token, float* out) {
    cudaStream_t s = m->ctx->stream;
    LSX_K(launch_take_row(s, m->embedding->data, m->embedding->kind, token, m->graph.hidden, out), "take_row");
    if (m->graph.embedding_scale != 1.f)
        LSX_K(launch_combine(s, out, out, m->graph.embedding_scale - 1.f, m->graph.hidden, out), "vector_sum");
    return LSX_OK;
}

int device_argmax(lsx_model* m, const float* z, size_t n, uint32_t* token, bool* nonfinite) {
    cudaStream_t s = m->ctx->stream;
    LSX_K(cudaMemsetAsync(m->d_best, 0, 8, s), "memset");
    LSX_K(cudaMemsetAsync(m->d_flag, 0, 4, s), "memset");
    argmax_kernel<<<std::min<size_t>(1024, (n + 255) / 256), 256, 0, s>>>(z, (int)n, m->d_best, m->d_flag);
    LSX_K(cudaGetLastError(), "argmax");
    unsigned long long best = 0;
    int flag = 0;
    LSX_K(cudaMemcpyAsync(&best, m->d_best, 8, cudaMemcpyDeviceToHost, s), "copy");
    LSX_K(cudaMemcpyAsync(&flag, m->d_flag, 4, cudaMemcpyDeviceToHost, s), "copy");
    LSX_K(cudaStreamSynchronize(s), "synchronize");
    *token = 0xffffffffu - (uint32_t)(best & 0xffffffffull);
    *nonfinite = flag != 0;
    return LSX_OK;
}

int read_device(lsx_model* m, float* host, const float* dev, size_t count) {
    LSX_K(cudaMemcpyAsync(host, dev, count * 4, cudaMemcpyDeviceToHost, m->ctx->stream), "device to host copy");
    return LSX_OK;
}

bool all_finite(const float* x, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(x[i])) return false;
    return true;
}

// One step of the per-op plan from the current residual buffer; returns the Frame.
int step_ops(lsx_model* m, const lsx_rotation* rotation, float* hidden_out, float* logits_out, uint32_t* argmax_out) {
    float* logits = nullptr;
    LSX_TRY(decode_ops(m, rotation, &logits));
    OpBuffers b = buffers_of(m);
    std::vector<float> hid(m->graph.hidden);
    LSX_TRY(read_device(m, hid.data(), b.hidden, m->graph.hidden));
    uint32_t token = 0;
    bool bad = false;
    LSX_TRY(device_argmax(m, logits, m->graph.vocab, &token, &bad));
    m->cursor += 1;
    if (bad || !all_finite(hid.data(), hid.size()))
        return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
    if (hidden_out) memcpy(hidden_out, hid.data(), hid.size() * 4);
    if (logits_out) {
        LSX_TRY(read_device(m, logits_out, logits, m->graph.vocab));
        LSX_K(cudaStreamSynchronize(m->ctx->stream), "synchronize");
    }
    if (argmax_out) *argmax_out = token;
    return LSX_OK;
}

// ----------------------------------------------------------- fused plan ----
int ensure_frames(lsx_model* m, size_t tokens) {
    if (tokens <= m->frames_capacity) return LSX_OK;
    if (m->d_frames) cudaFree(m->d_frames);
    m->d_frames = nullptr;
    m->frames_capacity = 0;
    size_t per = m->graph.hidden + m->graph.vocab;
    LSX_K(cudaMalloc(&m->d_frames, tokens * per * 4), "frame buffer allocation");
    m->frames_capacity = tokens;
    return LSX_OK;
}

void fill_rotation(DecodeState* st, const lsx_rotation* r) {
    st->rot_kind = 0;
    if (!r) return;
    if (!r->joint) {
        st->rot_kind = 1;
        st->rot_a = r->cosine_minus_one;
        st->rot_b = r->sine;
        st->rot_u = (const float*)r->u->data;
        st->rot_v = (const float*)r->v->data;
    } else {
        st->rot_kind = 2;
        st->rot_rank = (int)r->rank;
        st->rot_basis = (const float*)r->basis->data;
        st->rot_delta = (const float*)r->delta->data;
    }
}

// Runs `steps` fused decode steps under the state in m->host_state; reads the
// state back.
int run_fused(lsx_model* m, int steps) {
    cudaStream_t s = m->ctx->stream;
    DecodeState* dev = m->persistent ? m->persistent->state() : m->decoder->state();
    m->host_state->epoch = m->epoch;
    // Failure-path test hook of the persistent engine: LSX_DECODE_FAULT_TEST =
    // "cta,step,cycles" makes CTA `cta` withhold its argmax partial at `step` and
    // caps every exchange wait at `cycles` clock cycles, so the run ends with a
    // device status instead of output (no fault: only bounded waits expire).
    m->host_state->hold_cta = 0;
    m->host_state->hold_step = 0;
    m->host_state->spin_limit = 0;
    if (const char* v = getenv("LSX_DECODE_FAULT_TEST")) {
        int cta = -1, step = 0;
        long long cycles = 0;
        if (sscanf(v, "%d,%d,%lld", &cta, &step, &cycles) == 3 && cta >= 0 && step >= 0 && cycles > 0) {
            m->host_state->hold_cta = cta + 1;
            m->host_state->hold_step = step;
            m->host_state->spin_limit = cycles;
        }
    }
    LSX_K(cudaMemcpyAsync(dev, m->host_state, sizeof(DecodeState), cudaMemcpyHostToDevice, s), "state upload");
    if (m->persistent) LSX_TRY(m->persistent->run(steps));
    else LSX_TRY(m->decoder->enqueue_steps(steps));
    LSX_K(cudaMemcpyAsync(m->host_state, dev, sizeof(DecodeState), cudaMemcpyDeviceToHost, s), "state download");
    LSX_K(cudaStreamSynchronize(s), "decode");
    if (m->persistent) m->epoch = m->host_state->epoch;
    if (m->host_state->status != 0) {
        // A failed run may have published epochs it did not report: skip far past them.
        m->epoch += 1u << 24;
    }
    if (m->host_state->status != 0)
        return fail(LSX_E_CUDA, "decode kernel reported status " + std::to_string(m->host_state->status));
    return LSX_OK;
}

void base_state(lsx_model* m, const lsx_rotation* rotation) {
    DecodeState* st = m->host_state;
    memset(st, 0, sizeof(DecodeState));
    st->position = (int)m->cursor;
    st->prompt = m->d_prompt;
    st->tokens_out = m->d_tokens;
    st->inject = m->d_inject;
    st->hidden_scratch = m->d_hidden1;
    st->logits_scratch = m->d_logits1;
    fill_rotation(st, rotation);
}

int ensure_batched(lsx_model* m) {
    if (!m->batched) {
        std::unique_ptr<BatchedScorer> b(new BatchedScorer);
        LSX_TRY(b->build(m->ctx, m->fused_config, m->fused_layers));
        m->batched = std::move(b);
    }
    return LSX_OK;
}

// Prompts at least this long (less the last token) are prefilled in one batched
// forward; LSX_PREFILL_MIN overrides, 0 feeds every prompt token by token.
size_t batched_prefill_min() {
    const char* v = getenv("LSX_PREFILL_MIN");
    return v ? (size_t)std::max(0, atoi(v)) : 64;
}

int check_rotation(lsx_model* m, const lsx_rotation* rotation) {
    if (rotation) {
        LSX_ENSURE(rotation->ctx == m->ctx, "the rotation belongs to another context");
        LSX_ENSURE(rotation->width == m->graph.hidden, "the rotation width does not match the model");
    }
    return LSX_OK;
}

int single_fused(lsx_model* m, int mode, uint32_t token, const float* vector, const lsx_rotation* rotation,
                 float* hidden_out, float* logits_out, uint32_t* argmax_out) {
    cudaStream_t s = m->ctx->stream;
    if (mode == 0) LSX_K(cudaMemcpyAsync(m->d_prompt, &token, 4, cudaMemcpyHostToDevice, s), "token upload");
    else LSX_K(cudaMemcpyAsync(m->d_inject, vector, m->graph.hidden * 4, cudaMemcpyHostToDevice, s), "inject upload");
    base_state(m, rotation);
    DecodeState* st = m->host_state;
    st->mode = mode;
    st->prompt_length = 1;
    st->maximum = 1;
    LSX_TRY(run_fused(m, 1));
    m->cursor += 1;
    std::vector<float> hid(m->graph.hidden);
    LSX_K(cudaMemcpyAsync(hid.data(), m->d_hidden1, hid.size() * 4, cudaMemcpyDeviceToHost, s), "copy");
    if (logits_out)
        LSX_K(cudaMemcpyAsync(logits_out, m->d_logits1, m->graph.vocab * 4, cudaMemcpyDeviceToHost, s), "copy");
    LSX_K(cudaStreamSynchronize(s), "copy");
    if (m->host_state->nonfinite || !all_finite(hid.data(), hid.size()))
        return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
    if (hidden_out) memcpy(hidden_out, hid.data(), hid.size() * 4);
    if (argmax_out) *argmax_out = m->host_state->argmax;
    return LSX_OK;
}

}  // namespace

extern "C" {

int lsx_model_load(lsx_ctx* ctx, const char* root, size_t capacity, lsx_model** out) {
    LSX_ENSURE(ctx && root && out, "invalid argument");
    cudaSetDevice(ctx->device);
    Checkpoint ck;
    GraphSpec g;
    try {
        open_checkpoint(root, ck);
        std::string graph_path = std::string(root) + "/laplace.graph.json";
        if (is_file(graph_path)) g = from_graph_json(json::parse(read_text(graph_path)));
        else g = from_config(json::parse(read_text(std::string(root) + "/config.json")), ck);
        validate(g, ck);
    } catch (const std::exception& e) {
        return fail(LSX_E_FORMAT, e.what());
    }
    LSX_ENSURE(capacity > 0 && capacity <= g.max_context && capacity <= 2147483647ull,
               "check the execution context range");
    std::unique_ptr<lsx_model> m(new lsx_model);
    m->ctx = ctx;
    m->graph = g;
    m->capacity = capacity;
    for (auto& kv : ck.entries) m->parameters += kv.second.count();
    m->tensors = ck.entries.size();
    // LSX_DECODE_PLAN=ops selects the per-op plan for any checkpoint (used to
    // cross-check the two plans against each other).
    const char* plan = getenv("LSX_DECODE_PLAN");
    m->fused = fusable(g, ck) && !(plan && std::string(plan) == "ops");
    try {
        LSX_TRY(bank_take(m.get(), ck, g.embedding, &m->embedding));
        for (auto& S : g.blocks) {
            lsx_model::Block B;
            size_t qw = S.qheads * S.head_dim, kw = S.kvheads * S.head_dim;
            size_t length = capacity * kw;
            LSX_ENSURE(length <= 2147483647ull, "check the KV index range");
            LSX_TRY(bind_norm(m.get(), ck, S.input, 1, g.hidden, &B.input));
            LSX_TRY(bind_norm(m.get(), ck, S.post, 1, g.hidden, &B.post));
            bool upload = !m->fused;
            LSX_TRY(bind_proj(m.get(), ck, S.q, g.hidden, qw, upload, &B.q));
            LSX_TRY(bind_proj(m.get(), ck, S.k, g.hidden, kw, upload, &B.k));
            LSX_TRY(bind_proj(m.get(), ck, S.v, g.hidden, kw, upload, &B.v));
            LSX_TRY(bind_proj(m.get(), ck, S.o, qw, g.hidden, true, &B.o));
            B.has_qn = S.has_qn;
            B.has_kn = S.has_kn;
            if (S.has_qn) LSX_TRY(bind_norm(m.get(), ck, S.qn, S.qheads, S.head_dim, &B.qn));
            if (S.has_kn) LSX_TRY(bind_norm(m.get(), ck, S.kn, S.kvheads, S.head_dim, &B.kn));
            LSX_TRY(bind_proj(m.get(), ck, S.gate, g.hidden, S.intermediate, upload, &B.gate));
            LSX_TRY(bind_proj(m.get(), ck, S.up, g.hidden, S.intermediate, upload, &B.up));
            LSX_TRY(bind_proj(m.get(), ck, S.down, S.intermediate, g.hidden, true, &B.down));
            LSX_TRY(lsx_zeros(ctx, length, &B.keys));
            m->owned.push_back(B.keys);
            LSX_TRY(lsx_zeros(ctx, length, &B.values));
            m->owned.push_back(B.values);
            m->blocks.push_back(B);
        }
        LSX_TRY(bind_norm(m.get(), ck, g.final_norm, 1, g.hidden, &m->final_norm));
        LSX_TRY(bind_proj(m.get(), ck, g.readout, g.hidden, g.vocab, true, &m->head));
        LSX_K(cudaMalloc(&m->d_prompt, capacity * 4), "prompt buffer");
        LSX_K(cudaMalloc(&m->d_tokens, capacity * 4), "token buffer");
        LSX_K(cudaMalloc(&m->d_inject, g.hidden * 4), "inject buffer");
        LSX_K(cudaMalloc(&m->d_hidden1, g.hidden * 4), "hidden buffer");
        LSX_K(cudaMalloc(&m->d_logits1, g.vocab * 4), "logits buffer");
        LSX_K(cudaMalloc(&m->d_best, 8), "argmax buffer");
        LSX_K(cudaMalloc(&m->d_flag, 4), "flag buffer");
        LSX_K(cudaHostAlloc(&m->host_state, sizeof(DecodeState), cudaHostAllocDefault), "state staging");
        if (m->fused) {
            const BlockSpec& S0 = g.blocks[0];
            std::vector<FusedLayer> layers;
            for (size_t l = 0; l < g.blocks.size(); ++l) {
                const BlockSpec& S = g.blocks[l];
                lsx_model::Block& B = m->blocks[l];
                FusedLayer L{};
                size_t qw = S.qheads * S.head_dim, kw = S.kvheads * S.head_dim;
                lsx_tensor* t = nullptr;
                LSX_TRY(upload_rows(m.get(),
                                    {{&ck.entries.at(S.q.weight), qw},
                                     {&ck.entries.at(S.k.weight), kw},
                                     {&ck.entries.at(S.v.weight), kw}},
                                    g.hidden * 2, false, &t));
                L.wqkv = (const __nv_bfloat16*)t->data;
                LSX_TRY(upload_rows(m.get(),
                                    {{&ck.entries.at(S.gate.weight), S.intermediate},
                                     {&ck.entries.at(S.up.weight), S.intermediate}},
                                    g.hidden * 2, true, &t));
                L.wgu = (const __nv_bfloat16*)t->data;
                L.wo = (const __nv_bfloat16*)B.o.weight->data;
                L.wd = (const __nv_bfloat16*)B.down.weight->data;
                lsx_tensor* bias = nullptr;
                LSX_TRY(concat_bias(m.get(), ck, {{S.q.bias, qw}, {S.k.bias, kw}, {S.v.bias, kw}}, false, &bias));
                L.bqkv = bias ? (const float*)bias->data : nullptr;
                LSX_TRY(concat_bias(m.get(), ck, {{S.gate.bias, S.intermediate}, {S.up.bias, S.intermediate}}, true,
                                    &bias));
                L.bgu = bias ? (const float*)bias->data : nullptr;
                L.bo = B.o.bias ? (const float*)B.o.bias->data : nullptr;
                L.bd = B.down.bias ? (const float*)B.down.bias->data : nullptr;
                L.input_gain = (const float*)B.input.gain->data;
                L.post_gain = (const float*)B.post.gain->data;
                L.q_gain = B.has_qn ? (const float*)B.qn.gain->data : nullptr;
                L.k_gain = B.has_kn ? (const float*)B.kn.gain->data : nullptr;
                L.keys = (float*)B.keys->data;
                L.values = (float*)B.values->data;
                layers.push_back(L);
            }
            FusedConfig c{};
            c.hidden = (int)g.hidden;
            c.vocab = (int)g.vocab;
            c.layers = (int)g.blocks.size();
            c.qheads = (int)S0.qheads;
            c.kvheads = (int)S0.kvheads;
            c.head_dim = (int)S0.head_dim;
            c.intermediate = (int)S0.intermediate;
            c.rotary = (int)S0.rotary;
            c.interleaved = S0.interleaved ? 1 : 0;
            c.activation = S0.activation;
            c.capacity = (int)capacity;
            c.eps = S0.input.epsilon;
            c.qk_eps = S0.has_qn ? S0.qn.epsilon : (S0.has_kn ? S0.kn.epsilon : S0.input.epsilon);
            c.scale = S0.scale;
            c.embedding_scale = g.embedding_scale;
            c.theta = (double)S0.theta;
            c.embedding = m->embedding->data;
            c.embedding_kind = m->embedding->kind;
            c.head = (const __nv_bfloat16*)m->head.weight->data;
            c.head_bias = m->head.bias ? (const float*)m->head.bias->data : nullptr;
            c.final_gain = (const float*)m->final_norm.gain->data;
            m->fused_config = c;
            m->fused_layers = layers;
            std::string why;
            const char* engine = getenv("LSX_DECODE_ENGINE");  // "graph" selects the PDL kernel chain
            const bool want_persistent = !(engine && std::string(engine) == "graph");
            const bool debug = getenv("LSX_DEBUG") != nullptr;
            if (want_persistent && PersistentDecoder::eligible(c, ctx, &why)) {
                m->persistent.reset(new PersistentDecoder);
                if (m->persistent->build(ctx, c, layers) != LSX_OK) {
                    if (debug) fprintf(stderr, "[lsx] persistent decode engine not used: %s\n", lsx_last_error());
                    m->persistent.reset();
                }
            } else if (want_persistent && debug) {
                fprintf(stderr, "[lsx] persistent decode engine not eligible: %s\n", why.c_str());
            }
            if (!m->persistent) {
                if (FusedDecoder::eligible(c, &why)) {
                    m->decoder.reset(new FusedDecoder);
                    LSX_TRY(m->decoder->build(ctx, c, layers));
                } else {
                    m->fused = false;
                }
            }
        }
        if (!m->fused) {
            // The per-op plan needs every projection in the bank.
            for (size_t l = 0; l < g.blocks.size(); ++l) {
                const BlockSpec& S = g.blocks[l];
                lsx_model::Block& B = m->blocks[l];
                if (!B.q.weight) LSX_TRY(bank_take(m.get(), ck, S.q.weight, &B.q.weight));
                if (!B.k.weight) LSX_TRY(bank_take(m.get(), ck, S.k.weight, &B.k.weight));
                if (!B.v.weight) LSX_TRY(bank_take(m.get(), ck, S.v.weight, &B.v.weight));
                if (!B.gate.weight) LSX_TRY(bank_take(m.get(), ck, S.gate.weight, &B.gate.weight));
                if (!B.up.weight) LSX_TRY(bank_take(m.get(), ck, S.up.weight, &B.up.weight));
            }
        }
        OpBuffers ob;
        LSX_TRY(op_buffers(m.get(), &ob));
        LSX_K(cudaStreamSynchronize(ctx->stream), "model load");
    } catch (const std::exception& e) {
        return fail(LSX_E_FORMAT, e.what());
    }
    *out = m.release();
    return LSX_OK;
}

int lsx_model_free(lsx_model* model) {
    delete model;
    return LSX_OK;
}

int lsx_model_info_get(const lsx_model* m, lsx_model_info* out) {
    LSX_ENSURE(m && out, "invalid argument");
    memset(out, 0, sizeof(*out));
    const BlockSpec& b = m->graph.blocks[0];
    out->hidden_size = m->graph.hidden;
    out->vocab_size = m->graph.vocab;
    out->layers = m->graph.blocks.size();
    out->capacity = m->capacity;
    out->position = m->cursor;
    out->query_heads = b.qheads;
    out->kv_heads = b.kvheads;
    out->head_dim = b.head_dim;
    out->intermediate_size = b.intermediate;
    out->rotary_dim = b.rotary;
    out->parameters = m->parameters;
    out->tensors = m->tensors;
    out->eos_count = std::min<size_t>(8, m->graph.eos.size());
    for (size_t i = 0; i < out->eos_count; ++i) out->eos_token_ids[i] = m->graph.eos[i];
    out->fused = m->fused ? 1 : 0;
    out->graph = (m->decoder && m->decoder->supports_graph()) ? 1 : 0;
    out->kernels_per_step = m->decoder ? (uint64_t)m->decoder->kernels_per_step() : 0;
    out->persistent = m->persistent ? 1 : 0;
    return LSX_OK;
}

// Returns 1 when the fused decode plan runs this model, 0 for the per-op plan.
int lsx_model_fused(const lsx_model* m) { return m && m->fused ? 1 : 0; }

int lsx_model_reset(lsx_model* m) {
    LSX_ENSURE(m, "invalid argument");
    m->cursor = 0;
    return LSX_OK;
}

int lsx_model_rewind(lsx_model* m, size_t position) {
    LSX_ENSURE(m, "invalid argument");
    LSX_ENSURE(position <= m->cursor, "KV rewind must stay within the observed prefix");
    m->cursor = position;
    return LSX_OK;
}

int lsx_model_advance(lsx_model* m, uint32_t token, const lsx_rotation* rotation, float* hidden_out,
                      float* logits_out, uint32_t* argmax_out) {
    LSX_ENSURE(m, "invalid argument");
    LSX_ENSURE(token < m->graph.vocab && m->cursor < m->capacity, "check the token and context range");
    LSX_TRY(check_rotation(m, rotation));
    cudaSetDevice(m->ctx->device);
    if (m->fused) return single_fused(m, 0, token, nullptr, rotation, hidden_out, logits_out, argmax_out);
    OpBuffers b = buffers_of(m);
    LSX_TRY(embedding_into(m, token, b.residual));
    return step_ops(m, rotation, hidden_out, logits_out, argmax_out);
}

int lsx_model_inject(lsx_model* m, const float* vector, const lsx_rotation* rotation, float* hidden_out,
                     float* logits_out, uint32_t* argmax_out) {
    LSX_ENSURE(m && vector, "invalid argument");
    LSX_ENSURE(all_finite(vector, m->graph.hidden) && m->cursor < m->capacity,
               "check the injected vector width, finiteness and context");
    LSX_TRY(check_rotation(m, rotation));
    cudaSetDevice(m->ctx->device);
    if (m->fused) return single_fused(m, 1, 0, vector, rotation, hidden_out, logits_out, argmax_out);
    OpBuffers b = buffers_of(m);
    LSX_K(cudaMemcpyAsync(b.residual, vector, m->graph.hidden * 4, cudaMemcpyHostToDevice, m->ctx->stream),
          "inject upload");
    return step_ops(m, rotation, hidden_out, logits_out, argmax_out);
}

int lsx_model_embedding_vector(lsx_model* m, uint32_t token, float* out) {
    LSX_ENSURE(m && out, "invalid argument");
    LSX_ENSURE(token < m->graph.vocab, "check the embedding row range");
    cudaSetDevice(m->ctx->device);
    OpBuffers b = buffers_of(m);
    LSX_TRY(embedding_into(m, token, b.t));
    LSX_TRY(read_device(m, out, b.t, m->graph.hidden));
    LSX_K(cudaStreamSynchronize(m->ctx->stream), "synchronize");
    return LSX_OK;
}

int lsx_model_readout(lsx_model* m, const float* hidden, const lsx_rotation* rotation, float* logits_out) {
    LSX_ENSURE(m && hidden && logits_out, "invalid argument");
    LSX_ENSURE(all_finite(hidden, m->graph.hidden), "check the readout input width and finiteness");
    LSX_TRY(check_rotation(m, rotation));
    cudaSetDevice(m->ctx->device);
    OpBuffers b = buffers_of(m);
    cudaStream_t s = m->ctx->stream;
    LSX_K(cudaMemcpyAsync(b.hidden, hidden, m->graph.hidden * 4, cudaMemcpyHostToDevice, s), "upload");
    const float* input = b.hidden;
    if (rotation) {
        LSX_TRY(apply_rotation(m->ctx, rotation, b.hidden, b.rotated, b.norm, b.t, b.proj));
        input = b.rotated;
    }
    LSX_TRY(run_proj(m, m->head, input, b.logits));
    LSX_TRY(read_device(m, logits_out, b.logits, m->graph.vocab));
    LSX_K(cudaStreamSynchronize(s), "synchronize");
    if (!all_finite(logits_out, m->graph.vocab)) return fail(LSX_E_NONFINITE, "check the finiteness of the scores");
    return LSX_OK;
}

int lsx_model_head_image(lsx_model* m, const double* vector, float* out) {
    LSX_ENSURE(m && vector && out, "invalid argument");
    std::vector<float> v(m->graph.hidden);
    for (size_t i = 0; i < v.size(); ++i) {
        LSX_ENSURE(std::isfinite(vector[i]), "check the readout direction dimension");
        v[i] = (float)vector[i];
    }
    cudaSetDevice(m->ctx->device);
    OpBuffers b = buffers_of(m);
    cudaStream_t s = m->ctx->stream;
    LSX_K(cudaMemcpyAsync(b.rotated, v.data(), v.size() * 4, cudaMemcpyHostToDevice, s), "upload");
    LSX_TRY(run_proj(m, m->head, b.rotated, b.logits, false));
    LSX_TRY(read_device(m, out, b.logits, m->graph.vocab));
    LSX_K(cudaStreamSynchronize(s), "synchronize");
    return LSX_OK;
}

int lsx_model_head_images(lsx_model* m, const double* vectors, size_t count, float* out) {
    LSX_ENSURE(m && vectors && out && count > 0, "invalid argument");
    const size_t H = m->graph.hidden, V = m->graph.vocab;
    std::vector<float> v(count * H);
    for (size_t i = 0; i < v.size(); ++i) {
        LSX_ENSURE(std::isfinite(vectors[i]), "check the readout direction dimension");
        v[i] = (float)vectors[i];
    }
    if (m->head.weight->kind != LSX_BF16 || H % 8 != 0) {  // one matvec per direction
        for (size_t k = 0; k < count; ++k) LSX_TRY(lsx_model_head_image(m, vectors + k * H, out + k * V));
        return LSX_OK;
    }
    cudaSetDevice(m->ctx->device);
    const size_t out_bytes = (count * V * 4 + 255) & ~size_t(255);
    void* block = nullptr;
    LSX_TRY(device_alloc(m->ctx, out_bytes + head_images_scratch(count, H), &block));
    float* d_out = (float*)block;
    int rc = head_images_enqueue(m->ctx, m->head.weight, V, H, v.data(), count, d_out, (uint8_t*)block + out_bytes);
    if (rc == LSX_OK) {
        cudaError_t e = cudaMemcpyAsync(out, d_out, count * V * 4, cudaMemcpyDeviceToHost, m->ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(m->ctx->stream);
        if (e != cudaSuccess) rc = fail(LSX_E_CUDA, cuda_message("head images", e));
    }
    device_release(m->ctx, block);
    return rc;
}

int lsx_model_head_row(lsx_model* m, uint32_t token, float* out) {
    LSX_ENSURE(m && out, "invalid argument");
    LSX_ENSURE(token < m->graph.vocab, "check the output token range");
    cudaSetDevice(m->ctx->device);
    OpBuffers b = buffers_of(m);
    LSX_K(launch_take_row(m->ctx->stream, m->head.weight->data, m->head.weight->kind, token, m->graph.hidden, b.t),
          "take_row");
    LSX_TRY(read_device(m, out, b.t, m->graph.hidden));
    LSX_K(cudaStreamSynchronize(m->ctx->stream), "synchronize");
    return LSX_OK;
}

int lsx_model_head(lsx_model* m, const lsx_tensor** weight, const lsx_tensor** bias) {
    LSX_ENSURE(m && weight, "invalid argument");
    *weight = m->head.weight;
    if (bias) *bias = m->head.bias;
    return LSX_OK;
}

int lsx_model_generate(lsx_model* m, const uint32_t* prompt, size_t prompt_length, size_t maximum,
                       const uint32_t* stop_tokens, size_t stop_count, const lsx_rotation* rotation,
                       uint32_t* tokens_out, size_t* generated, int* stopped, float* hidden_frames,
                       float* logits_frames) {
    LSX_ENSURE(m && prompt && tokens_out && generated, "invalid argument");
    // generate_frames (src/diagnosis.rs:106-121) and prefill (src/diagnosis.rs:81-99)
    LSX_ENSURE(maximum > 0 && prompt_length + maximum <= m->capacity,
               "give a context that fits the input and generation length");
    LSX_ENSURE(prompt_length > 0 && prompt_length <= m->capacity, "check the input token length");
    for (size_t i = 0; i < prompt_length; ++i) LSX_ENSURE(prompt[i] < m->graph.vocab, "check the token range");
    LSX_ENSURE(stop_count <= 16 && (stop_count == 0 || stop_tokens), "at most 16 stop tokens");
    LSX_TRY(check_rotation(m, rotation));
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    m->cursor = 0;  // prefill starts with model.reset()
    const size_t H = m->graph.hidden, V = m->graph.vocab;
    const bool want_frames = hidden_frames || logits_frames;
    if (m->fused) {
        if (want_frames) LSX_TRY(ensure_frames(m, maximum));
        // A long prompt: all but its last token in one batched forward that fills
        // the KV cache, then the decode engine continues from the last token.
        size_t skip = 0;
        const size_t min_batch = batched_prefill_min();
        if (min_batch > 0 && prompt_length - 1 >= min_batch && BatchedScorer::eligible(m->fused_config, nullptr)) {
            LSX_TRY(ensure_batched(m));
            LSX_TRY(m->batched->prefill(prompt, prompt_length - 1));
            skip = prompt_length - 1;
            m->cursor = skip;
        }
        LSX_K(cudaMemcpyAsync(m->d_prompt, prompt + skip, (prompt_length - skip) * 4, cudaMemcpyHostToDevice, s),
              "prompt upload");
        base_state(m, rotation);
        DecodeState* st = m->host_state;
        st->prompt_length = (int)(prompt_length - skip);
        st->maximum = (int)maximum;
        st->n_stop = (int)stop_count;
        for (size_t i = 0; i < stop_count; ++i) st->stop[i] = stop_tokens[i];
        if (want_frames) {
            st->frames = 1;
            st->hidden_frames = m->d_frames;
            st->logits_frames = m->d_frames + maximum * H;
        }
        LSX_TRY(run_fused(m, (int)(prompt_length - skip + maximum - 1)));
        size_t n = (size_t)m->host_state->generated;
        LSX_K(cudaMemcpyAsync(tokens_out, m->d_tokens, n * 4, cudaMemcpyDeviceToHost, s), "token download");
        if (hidden_frames)
            LSX_K(cudaMemcpyAsync(hidden_frames, m->d_frames, n * H * 4, cudaMemcpyDeviceToHost, s), "frames");
        if (logits_frames) LSX_TRY(staged_download(m->ctx, logits_frames, m->d_frames + maximum * H, n * V * 4));
        LSX_K(cudaStreamSynchronize(s), "generate");
        if (m->host_state->nonfinite) return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
        *generated = n;
        m->cursor = (size_t)m->host_state->position;
        bool stop = false;
        if (n > 0)
            for (size_t i = 0; i < stop_count; ++i) stop |= stop_tokens[i] == tokens_out[n - 1];
        if (stopped) *stopped = stop ? 1 : 0;
        return LSX_OK;
    }
    // Per-op plan: the reference's host loop.
    uint32_t next = 0;
    std::vector<float> hid(H), logits(want_frames ? V : 0);
    for (size_t i = 0; i < prompt_length; ++i) {
        OpBuffers b = buffers_of(m);
        LSX_TRY(embedding_into(m, prompt[i], b.residual));
        LSX_TRY(step_ops(m, rotation, hid.data(), want_frames ? logits.data() : nullptr, &next));
    }
    size_t n = 0;
    bool stop = false;
    for (size_t position = 0; position < maximum; ++position) {
        tokens_out[n] = next;
        if (hidden_frames) memcpy(hidden_frames + n * H, hid.data(), H * 4);
        if (logits_frames) memcpy(logits_frames + n * V, logits.data(), V * 4);
        ++n;
        for (size_t i = 0; i < stop_count; ++i) stop |= stop_tokens[i] == next;
        if (stop || position + 1 == maximum) break;
        OpBuffers b = buffers_of(m);
        LSX_TRY(embedding_into(m, next, b.residual));
        LSX_TRY(step_ops(m, rotation, hid.data(), want_frames ? logits.data() : nullptr, &next));
    }
    *generated = n;
    if (stopped) *stopped = stop ? 1 : 0;
    return LSX_OK;
}

// Teacher-forced scoring of one case (src/scaling.rs:181-216): prefill the prompt,
// then for each target score the frame that predicts it and advance with the target.
int lsx_model_score(lsx_model* m, const uint32_t* prompt, size_t prompt_length, const uint32_t* targets,
                    size_t count, const lsx_rotation* rotation, double* nll_out, uint32_t* argmax_out,
                    float* hidden_frames, float* logits_frames) {
    LSX_ENSURE(m && prompt && targets, "invalid argument");
    LSX_ENSURE(prompt_length > 0 && count > 0 && prompt_length + count - 1 <= m->capacity,
               "give a context that fits the prompt and the continuation");
    for (size_t i = 0; i < prompt_length; ++i) LSX_ENSURE(prompt[i] < m->graph.vocab, "check the token range");
    for (size_t i = 0; i < count; ++i) LSX_ENSURE(targets[i] < m->graph.vocab, "check the target range");
    LSX_TRY(check_rotation(m, rotation));
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    m->cursor = 0;
    const size_t H = m->graph.hidden, V = m->graph.vocab;
    const size_t forced = prompt_length + count - 1;  // prompt, then every target but the last
    if (m->fused) {
        LSX_TRY(ensure_frames(m, count));
        std::vector<uint32_t> seq(forced);
        memcpy(seq.data(), prompt, prompt_length * 4);
        if (count > 1) memcpy(seq.data() + prompt_length, targets, (count - 1) * 4);
        void* block = nullptr;
        LSX_TRY(device_alloc(m->ctx, count * 12 + 16, &block));
        uint32_t* d_targets = (uint32_t*)block;
        double* d_nll = (double*)((uint8_t*)block + ((count * 4 + 15) & ~(size_t)15));
        int rc = LSX_OK;
        cudaError_t e = cudaMemcpyAsync(m->d_prompt, seq.data(), forced * 4, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_targets, targets, count * 4, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) rc = fail(LSX_E_CUDA, cuda_message("score upload", e));
        if (rc == LSX_OK) {
            base_state(m, rotation);
            DecodeState* st = m->host_state;
            st->prompt_length = (int)forced;
            st->maximum = (int)count;
            st->frame_back = (int)count - 1;
            st->frames = 1;
            st->hidden_frames = m->d_frames;
            st->logits_frames = m->d_frames + count * H;
            rc = run_fused(m, (int)forced);
        }
        if (rc == LSX_OK) {
            frame_nll_kernel<<<(int)count, 1024, 0, s>>>(m->d_frames + count * H, (int)V, d_targets, d_nll);
            e = cudaGetLastError();
            if (e == cudaSuccess && nll_out) e = cudaMemcpyAsync(nll_out, d_nll, count * 8, cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess && argmax_out)
                e = cudaMemcpyAsync(argmax_out, m->d_tokens, count * 4, cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess && hidden_frames)
                e = cudaMemcpyAsync(hidden_frames, m->d_frames, count * H * 4, cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) rc = fail(LSX_E_CUDA, cuda_message("score", e));
            if (rc == LSX_OK && logits_frames)
                rc = staged_download(m->ctx, logits_frames, m->d_frames + count * H, count * V * 4);
        }
        device_release(m->ctx, block);
        if (rc != LSX_OK) return rc;
        if (m->host_state->nonfinite) return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
        m->cursor = (size_t)m->host_state->position;
        return LSX_OK;
    }
    // Per-op plan: the reference's host loop, loss on the host in f64.
    std::vector<float> hid(H), logits(V);
    uint32_t next = 0;
    for (size_t i = 0; i < prompt_length; ++i) {
        OpBuffers b = buffers_of(m);
        LSX_TRY(embedding_into(m, prompt[i], b.residual));
        LSX_TRY(step_ops(m, rotation, hid.data(), i + 1 == prompt_length ? logits.data() : nullptr, &next));
    }
    for (size_t k = 0; k < count; ++k) {
        double top = -INFINITY, sum = 0.0;
        for (size_t j = 0; j < V; ++j) top = std::max(top, (double)logits[j]);
        for (size_t j = 0; j < V; ++j) sum += std::exp((double)logits[j] - top);
        if (nll_out) nll_out[k] = top + std::log(sum) - (double)logits[targets[k]];
        if (argmax_out) argmax_out[k] = next;
        if (hidden_frames) memcpy(hidden_frames + k * H, hid.data(), H * 4);
        if (logits_frames) memcpy(logits_frames + k * V, logits.data(), V * 4);
        if (k + 1 == count) break;
        OpBuffers b = buffers_of(m);
        LSX_TRY(embedding_into(m, targets[k], b.residual));
        LSX_TRY(step_ops(m, rotation, hid.data(), logits.data(), &next));
    }
    return LSX_OK;
}

// Teacher-forced scoring of many equal-length cases at once (the per-case loop of
// src/scaling.rs:181-216 batched over cases): every case's prompt and targets but
// the last go through the decoder together, one tensor-core GEMM per projection.
int lsx_model_generate_batch(lsx_model* m, const uint32_t* prompts, size_t batch, size_t prompt_length,
                             size_t maximum, uint32_t* tokens_out) {
    LSX_ENSURE(m && prompts && tokens_out, "invalid argument");
    LSX_ENSURE(batch > 0 && prompt_length >= 2 && maximum > 0,
               "give at least one sequence, two prompt tokens and one generated token");
    for (size_t i = 0; i < batch * prompt_length; ++i) LSX_ENSURE(prompts[i] < m->graph.vocab, "check the token range");
    if (!m->fused) return fail(LSX_E_UNSUPPORTED, "batched generation needs the fused weight layout");
    cudaSetDevice(m->ctx->device);
    LSX_TRY(ensure_batched(m));
    return m->batched->generate_batch(prompts, batch, prompt_length, maximum, tokens_out);
}

int lsx_model_score_batch(lsx_model* m, const uint32_t* prompts, size_t cases, size_t prompt_length,
                          const uint32_t* targets, size_t count, const lsx_rotation* rotation, double* nll_out,
                          uint32_t* argmax_out, double* margin_out, float* logits_out) {
    LSX_ENSURE(m && prompts && targets, "invalid argument");
    LSX_ENSURE(cases > 0 && prompt_length > 0 && count > 0, "give at least one case, prompt token and target");
    LSX_ENSURE(prompt_length + count - 1 <= m->capacity, "give a context that fits the prompt and the continuation");
    for (size_t i = 0; i < cases * prompt_length; ++i) LSX_ENSURE(prompts[i] < m->graph.vocab, "check the token range");
    for (size_t i = 0; i < cases * count; ++i) LSX_ENSURE(targets[i] < m->graph.vocab, "check the target range");
    if (!m->fused) return fail(LSX_E_UNSUPPORTED, "batched scoring needs the fused weight layout");
    LSX_TRY(check_rotation(m, rotation));
    cudaSetDevice(m->ctx->device);
    LSX_TRY(ensure_batched(m));
    const size_t T = prompt_length + count - 1;
    std::vector<uint32_t> fed(cases * T);
    for (size_t c = 0; c < cases; ++c) {
        memcpy(fed.data() + c * T, prompts + c * prompt_length, prompt_length * 4);
        if (count > 1) memcpy(fed.data() + c * T + prompt_length, targets + c * count, (count - 1) * 4);
    }
    BatchedScorer::Outputs out;
    out.nll = nll_out;
    out.argmax = argmax_out;
    out.margin = margin_out;
    out.logits = logits_out;
    return m->batched->score(fed.data(), cases, T, prompt_length - 1, count, targets, rotation, out);
}

}  // extern "C"
