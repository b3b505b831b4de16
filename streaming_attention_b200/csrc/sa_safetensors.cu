// sa_safetensors.cu -- Qwen3 weights from a safetensors checkpoint, uploaded
// without the fp32 round trip.
//
// Replaces load_qwen3_weights (tensor_cpp/src/qwen3_loader.cpp:140-297), which
// reads the file's tensors one by one through an ifstream, widens every bf16
// value to fp32 on the host and hands fp32 tensors to the model.  Here the
// file is memory-mapped and each weight goes from the mapped bytes to the
// GPU's packed bf16 layout in at most three 2-D copies; only the small norm
// gains are widened (to the fp32 the kernels use).
//
// Format (the public safetensors layout): an 8-byte little-endian header
// length N, N bytes of JSON mapping each tensor name to {"dtype", "shape",
// "data_offsets": [begin, end]} (offsets relative to the byte after the
// header; an optional "__metadata__" entry), then the data.  Names follow the
// Hugging Face Qwen3 checkpoint, as the reference loader reads them:
//   model.embed_tokens.weight [V, H], model.norm.weight [H],
//   lm_head.weight [V, H] (optional here: absent means tied to the embedding,
//   as Qwen3-0.6B's tie_word_embeddings; the reference loader requires it),
//   model.layers.{i}.{input_layernorm, post_attention_layernorm}.weight [H],
//   model.layers.{i}.self_attn.{q,k,v,o}_proj.weight, .{q,k}_norm.weight [D],
//   model.layers.{i}.mlp.{gate,up,down}_proj.weight.
// The configuration is inferred from the shapes (the reference hardcodes
// Qwen3-0.6B's: 28 layers, 16/8 heads, head_dim 128): layers counted from
// index 0, head_dim from q_norm, heads from q_proj / k_proj rows, inter from
// gate_proj.  Element types BF16 (the checkpoint's), F16 and F32 are accepted.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "sa_internal.h"
#include "sa_qwen3.h"

namespace sa {
namespace st {

// ---- a small JSON reader, enough for safetensors headers -------------------
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0.0;
    bool is_int = false;
    unsigned long long u = 0;   // the value when is_int and non-negative
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* key) const {
        for (auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* e;
    std::string err;
    int depth = 0;

    bool fail(const char* what) {
        if (err.empty()) err = what;
        return false;
    }
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool lit(const char* s) {
        const size_t n = std::strlen(s);
        if ((size_t)(e - p) < n || std::memcmp(p, s, n) != 0) return fail("bad literal");
        p += n;
        return true;
    }
    bool string(std::string& out) {
        if (p >= e || *p != '"') return fail("expected string");
        ++p;
        while (p < e && *p != '"') {
            char c = *p++;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p >= e) return fail("bad escape");
            c = *p++;
            switch (c) {
                case '"': case '\\': case '/': out += c; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {   // keep ASCII code points, others as '?': names are ASCII
                    if (e - p < 4) return fail("bad \\u escape");
                    unsigned cp = 0;
                    for (int i = 0; i < 4; ++i) {
                        const char h = *p++;
                        cp = cp * 16 + (h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                        : h >= 'A' && h <= 'F' ? h - 'A' + 10 : 99);
                        if (cp > 0xFFFF) return fail("bad \\u escape");
                    }
                    out += cp < 0x80 ? (char)cp : '?';
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool number(JVal& v) {
        const char* s = p;
        if (p < e && *p == '-') ++p;
        bool frac = false;
        while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-')) {
            if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
            ++p;
        }
        if (p == s) return fail("expected a value");
        const std::string tok(s, p);
        v.kind = JVal::NUM;
        v.num = std::strtod(tok.c_str(), nullptr);
        if (!frac && tok[0] != '-') {
            v.is_int = true;
            v.u = std::strtoull(tok.c_str(), nullptr, 10);
        }
        return true;
    }
    bool value(JVal& v) {
        if (++depth > 64) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        bool ok;
        if (*p == '{') {
            v.kind = JVal::OBJ;
            ++p;
            ws();
            ok = true;
            if (p < e && *p == '}') {
                ++p;
            } else {
                while (ok) {
                    std::string k;
                    ws();
                    if (!string(k)) { ok = false; break; }
                    ws();
                    if (p >= e || *p != ':') { ok = fail("expected ':'"); break; }
                    ++p;
                    v.obj.emplace_back(std::move(k), JVal());
                    if (!value(v.obj.back().second)) { ok = false; break; }
                    ws();
                    if (p < e && *p == ',') { ++p; continue; }
                    if (p < e && *p == '}') { ++p; break; }
                    ok = fail("expected ',' or '}'");
                }
            }
        } else if (*p == '[') {
            v.kind = JVal::ARR;
            ++p;
            ws();
            ok = true;
            if (p < e && *p == ']') {
                ++p;
            } else {
                while (ok) {
                    v.arr.emplace_back();
                    if (!value(v.arr.back())) { ok = false; break; }
                    ws();
                    if (p < e && *p == ',') { ++p; continue; }
                    if (p < e && *p == ']') { ++p; break; }
                    ok = fail("expected ',' or ']'");
                }
            }
        } else if (*p == '"') {
            v.kind = JVal::STR;
            ok = string(v.str);
        } else if (*p == 't') {
            v.kind = JVal::BOOL; v.b = true; ok = lit("true");
        } else if (*p == 'f') {
            v.kind = JVal::BOOL; ok = lit("false");
        } else if (*p == 'n') {
            ok = lit("null");
        } else {
            ok = number(v);
        }
        --depth;
        return ok;
    }
};

// ---- the file --------------------------------------------------------------
struct Tensor {
    int type = -1;                  // QW_SRC_*
    std::vector<size_t> shape;
    size_t begin = 0, end = 0;      // byte range within the data section
    size_t numel() const {
        size_t n = 1;
        for (size_t s : shape) n *= s;
        return n;
    }
};

struct File {
    int fd = -1;
    void* map = nullptr;
    size_t size = 0;
    const unsigned char* data = nullptr;   // start of the data section
    size_t data_size = 0;
    std::map<std::string, Tensor> tensors;
    std::vector<std::vector<unsigned char>> aligned;   // copies of misaligned tensors
    ~File() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
};

static int elem_size(int type) { return type == QW_SRC_F32 ? 4 : 2; }

static int open_file(const char* path, File& f) {
    SA_CHECK_ARG(path != nullptr, "safetensors: path is NULL");
    f.fd = open(path, O_RDONLY);
    if (f.fd < 0) return set_error(SA_ERR_ARG, "safetensors: cannot open %s", path);
    struct stat sb;
    if (fstat(f.fd, &sb) != 0) return set_error(SA_ERR_ARG, "safetensors: cannot stat %s", path);
    f.size = (size_t)sb.st_size;
    SA_CHECK_ARG(f.size >= 8, "safetensors: %s is shorter than its 8-byte header length", path);
    f.map = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
    if (f.map == MAP_FAILED) return set_error(SA_ERR_ARG, "safetensors: cannot map %s", path);
    const unsigned char* base = static_cast<const unsigned char*>(f.map);
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
    SA_CHECK_ARG(hlen <= f.size - 8 && hlen <= (100ull << 20),
                 "safetensors: header length %llu does not fit the file (%zu bytes)", (unsigned long long)hlen,
                 f.size);
    f.data = base + 8 + hlen;
    f.data_size = f.size - 8 - hlen;
    JParser jp{reinterpret_cast<const char*>(base + 8), reinterpret_cast<const char*>(base + 8 + hlen)};
    JVal root;
    if (!jp.value(root) || root.kind != JVal::OBJ)
        return set_error(SA_ERR_ARG, "safetensors: header is not a JSON object (%s)", jp.err.c_str());
    for (auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal& t = kv.second;
        const JVal* dt = t.get("dtype");
        const JVal* sh = t.get("shape");
        const JVal* off = t.get("data_offsets");
        SA_CHECK_ARG(t.kind == JVal::OBJ && dt && dt->kind == JVal::STR && sh && sh->kind == JVal::ARR && off &&
                         off->kind == JVal::ARR && off->arr.size() == 2,
                     "safetensors: entry %s lacks dtype / shape / data_offsets", kv.first.c_str());
        Tensor x;
        if (dt->str == "BF16") x.type = QW_SRC_BF16;
        else if (dt->str == "F16") x.type = QW_SRC_F16;
        else if (dt->str == "F32") x.type = QW_SRC_F32;
        for (const JVal& d : sh->arr) {
            SA_CHECK_ARG(d.is_int, "safetensors: %s has a non-integer dimension", kv.first.c_str());
            x.shape.push_back((size_t)d.u);
        }
        SA_CHECK_ARG(off->arr[0].is_int && off->arr[1].is_int, "safetensors: %s has bad data_offsets",
                     kv.first.c_str());
        x.begin = (size_t)off->arr[0].u;
        x.end = (size_t)off->arr[1].u;
        SA_CHECK_ARG(x.begin <= x.end && x.end <= f.data_size,
                     "safetensors: %s data [%zu, %zu) lies outside the %zu data bytes", kv.first.c_str(), x.begin,
                     x.end, f.data_size);
        if (x.type >= 0)
            SA_CHECK_ARG(x.end - x.begin == x.numel() * elem_size(x.type),
                         "safetensors: %s holds %zu bytes for %zu elements of %s", kv.first.c_str(),
                         x.end - x.begin, x.numel(), dt->str.c_str());
        f.tensors.emplace(kv.first, std::move(x));
    }
    return SA_OK;
}

// The named tensor with the expected shape, as an upload source.
static int source(File& f, const std::string& name, std::vector<size_t> shape, QwSrc* out) {
    auto it = f.tensors.find(name);
    SA_CHECK_ARG(it != f.tensors.end(), "safetensors: tensor %s not found", name.c_str());
    const Tensor& t = it->second;
    SA_CHECK_ARG(t.type >= 0, "safetensors: %s has an element type other than BF16, F16, F32", name.c_str());
    if (t.shape != shape) {
        std::string want, got;
        for (size_t s : shape) want += std::to_string(s) + " ";
        for (size_t s : t.shape) got += std::to_string(s) + " ";
        return set_error(SA_ERR_ARG, "safetensors: %s has shape [%s] where [%s] is expected", name.c_str(),
                         got.c_str(), want.c_str());
    }
    const unsigned char* p = f.data + t.begin;
    if (((uintptr_t)p % elem_size(t.type)) != 0) {   // keep element loads aligned
        f.aligned.emplace_back(p, p + (t.end - t.begin));
        p = f.aligned.back().data();
    }
    *out = QwSrc{p, t.type};
    return SA_OK;
}

static std::string layer_name(int i, const char* rest) { return "model.layers." + std::to_string(i) + "." + rest; }

// Infer the configuration from the tensor shapes.
static int infer_config(File& f, int max_seq, float eps, float theta, sa_qwen3_config* c) {
    auto it = f.tensors.find("model.embed_tokens.weight");
    SA_CHECK_ARG(it != f.tensors.end() && it->second.shape.size() == 2,
                 "safetensors: model.embed_tokens.weight [vocab, hidden] not found");
    std::memset(c, 0, sizeof(*c));
    c->vocab = (int)it->second.shape[0];
    c->hidden = (int)it->second.shape[1];
    int L = 0;
    while (f.tensors.count(layer_name(L, "input_layernorm.weight"))) ++L;
    SA_CHECK_ARG(L > 0, "safetensors: no model.layers.0.* tensors");
    c->n_layers = L;
    auto shp = [&](const std::string& n) -> const std::vector<size_t>* {
        auto t = f.tensors.find(n);
        return t == f.tensors.end() ? nullptr : &t->second.shape;
    };
    const auto* qn = shp(layer_name(0, "self_attn.q_norm.weight"));
    const auto* qp = shp(layer_name(0, "self_attn.q_proj.weight"));
    const auto* kp = shp(layer_name(0, "self_attn.k_proj.weight"));
    const auto* gp = shp(layer_name(0, "mlp.gate_proj.weight"));
    SA_CHECK_ARG(qn && qn->size() == 1 && qp && qp->size() == 2 && kp && kp->size() == 2 && gp && gp->size() == 2,
                 "safetensors: layer 0 lacks q_norm / q_proj / k_proj / gate_proj");
    c->head_dim = (int)(*qn)[0];
    SA_CHECK_ARG(c->head_dim > 0 && (*qp)[0] % c->head_dim == 0 && (*kp)[0] % c->head_dim == 0,
                 "safetensors: q_proj / k_proj rows are not multiples of head_dim %d", c->head_dim);
    c->hq = (int)((*qp)[0] / c->head_dim);
    c->hkv = (int)((*kp)[0] / c->head_dim);
    c->inter = (int)(*gp)[0];
    c->eps = eps > 0.f ? eps : 1e-6f;
    c->theta = theta > 0.f ? theta : 1000000.0f;
    c->max_seq = max_seq;
    return SA_OK;
}

// Every tensor the model needs, checked against the configuration.
struct Sources {
    QwSrc embed, norm, head{nullptr, QW_SRC_BF16};
    std::vector<std::vector<QwSrc>> layers;
};

static int collect(File& f, const sa_qwen3_config& c, Sources* s) {
    const size_t V = c.vocab, H = c.hidden, D = c.head_dim, I = c.inter;
    const size_t QD = (size_t)c.hq * D, KD = (size_t)c.hkv * D;
    SA_RC_TRY(source(f, "model.embed_tokens.weight", {V, H}, &s->embed));
    SA_RC_TRY(source(f, "model.norm.weight", {H}, &s->norm));
    if (f.tensors.count("lm_head.weight")) SA_RC_TRY(source(f, "lm_head.weight", {V, H}, &s->head));
    s->layers.assign(c.n_layers, std::vector<QwSrc>(11));
    for (int i = 0; i < c.n_layers; ++i) {
        auto& w = s->layers[i];
        auto N = [&](const char* r) { return layer_name(i, r); };
        SA_RC_TRY(source(f, N("input_layernorm.weight"), {H}, &w[0]));
        SA_RC_TRY(source(f, N("self_attn.q_proj.weight"), {QD, H}, &w[1]));
        SA_RC_TRY(source(f, N("self_attn.k_proj.weight"), {KD, H}, &w[2]));
        SA_RC_TRY(source(f, N("self_attn.v_proj.weight"), {KD, H}, &w[3]));
        SA_RC_TRY(source(f, N("self_attn.q_norm.weight"), {D}, &w[4]));
        SA_RC_TRY(source(f, N("self_attn.k_norm.weight"), {D}, &w[5]));
        SA_RC_TRY(source(f, N("self_attn.o_proj.weight"), {H, QD}, &w[6]));
        SA_RC_TRY(source(f, N("post_attention_layernorm.weight"), {H}, &w[7]));
        SA_RC_TRY(source(f, N("mlp.gate_proj.weight"), {I, H}, &w[8]));
        SA_RC_TRY(source(f, N("mlp.up_proj.weight"), {I, H}, &w[9]));
        SA_RC_TRY(source(f, N("mlp.down_proj.weight"), {H, I}, &w[10]));
    }
    return SA_OK;
}

}  // namespace st
}  // namespace sa

SA_API int sa_safetensors_inspect(const char* path, sa_qwen3_config* out) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(out != nullptr, "sa_safetensors_inspect: out is NULL");
    st::File f;
    SA_RC_TRY(st::open_file(path, f));
    sa_qwen3_config c;
    SA_RC_TRY(st::infer_config(f, 0, 0.f, 0.f, &c));
    st::Sources s;
    SA_RC_TRY(st::collect(f, c, &s));
    *out = c;
    return SA_OK;
}

SA_API int sa_qwen3_load_safetensors(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta,
                                     sa_qwen3** out) {
    return sa_qwen3_load_safetensors_tp(ctx, path, max_seq, eps, theta, 0, 1, out);
}

namespace sa {
// Create the model (head-parallel share, or with `sequence` a whole model of
// a sequence-parallel rank) and upload the checkpoint's tensors.
static int load_checkpoint(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta, int rank, int world,
                           bool sequence, sa_qwen3** out) {
    clear_error();
    SA_CHECK_ARG(ctx && out, "sa_qwen3_load_safetensors: null argument");
    *out = nullptr;
    SA_CHECK_ARG(max_seq > 0, "sa_qwen3_load_safetensors: max_seq=%d", max_seq);
    st::File f;
    SA_RC_TRY(st::open_file(path, f));
    sa_qwen3_config c;
    SA_RC_TRY(st::infer_config(f, max_seq, eps, theta, &c));
    st::Sources s;
    SA_RC_TRY(st::collect(f, c, &s));   // every tensor checked before the model is allocated
    sa_qwen3* m = nullptr;
    if (sequence)
        SA_RC_TRY(sa_qwen3_create_sp(ctx, &c, rank, world, &m));
    else
        SA_RC_TRY(qwen3_create_model(ctx, &c, rank, world, &m));
    int rc;
    {
        DeviceGuard guard(ctx->device);
        rc = qwen3_upload_embed(m, s.embed, s.norm, s.head);
        for (int i = 0; !rc && i < c.n_layers; ++i) {
            const auto& w = s.layers[i];
            rc = qwen3_upload_layer(m, i, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], w[8], w[9], w[10]);
        }
    }
    if (rc) {
        const std::string msg = sa_last_error();
        sa_qwen3_destroy(m);
        return set_error(rc, "%s", msg.c_str());
    }
    *out = m;
    return SA_OK;
}
}  // namespace sa

SA_API int sa_qwen3_load_safetensors_tp(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta, int rank,
                                        int world, sa_qwen3** out) {
    return sa::load_checkpoint(ctx, path, max_seq, eps, theta, rank, world, false, out);
}

SA_API int sa_qwen3_load_safetensors_sp(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta, int rank,
                                        int world, sa_qwen3** out) {
    return sa::load_checkpoint(ctx, path, max_seq, eps, theta, rank, world, true, out);
}
