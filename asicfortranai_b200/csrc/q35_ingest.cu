// q35_ingest.cu -- weight-file readers of the model runtime (host code).
//
//  * The stream-binary layer file of weight_loader.f90:18-182 (load_layer_weights), as
//    written by generate_test_weights.f90:154-183 and scripts/convert_weights_to_fortran.py
//    :94-121: for wq, wk, wv, wo, w_gate, w_up, w_down in that order, the packed INT4
//    matrix W_Q(K/2,N) column-major (N*K/2 bytes) followed by its scales[N] (fp32); the
//    Python converter appends attn_norm[hidden] and ffn_norm[hidden] (fp32).  Little endian.
//  * The 3.5-bit safetensors file of convert_weights_3p5bit.py:105-139: each quantized
//    matrix `key` is stored as `key.weight_q` (int8 [K/2][N], row-major as numpy writes
//    it), `key.scales` and `key.offsets` (fp32 [N]); tensors kept in floating point (norms,
//    and embeddings when not quantized) are fp16 (or fp32 / bf16).  Keys follow the
//    LLaMA checkpoint names: model.layers.{l}.self_attn.{q,k,v,o}_proj.weight,
//    model.layers.{l}.mlp.{gate,up,down}_proj.weight, model.layers.{l}.input_layernorm.weight,
//    model.layers.{l}.post_attention_layernorm.weight, model.embed_tokens.weight,
//    model.norm.weight, lm_head.weight.  A matrix is quantized as [K][N] = [input][output]
//    (quantize_3p5bit_asymmetric's contract: per output column n, K/2 pair bytes).  The
//    embedding [vocab][hidden] and the LM head [vocab][hidden] may be quantized too (the
//    converter quantizes every 2-D tensor): they are expanded as value = code * scale +
//    zero_point (the quantizer's inverse), code the 4-bit (even row) or 3-bit (odd row)
//    field of the pair byte.
// Both readers stream one tensor at a time through host memory into
// q35_model_set_layer / the embedding upload, which repack the reference bytes into the
// device tile format on the GPU (and keep each tensor-parallel rank's shard).
#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "q35_layer.cuh"

using namespace q35;

namespace {

// ---- a minimal JSON reader for the safetensors header ---------------------------------
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0.0;
    long long inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal *get(const std::string &k) const {
        for (const auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char *p, *e;
    std::string err;
    int depth = 0;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char *m) {
        if (err.empty()) err = m;
        return false;
    }
    bool str(std::string &out) {
        if (p >= e || *p != '"') return fail("expected a string");
        ++p;
        while (p < e && *p != '"') {
            if (*p == '\\') {
                if (++p >= e) return fail("bad escape");
                switch (*p) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {   // keep ASCII code points, replace the rest
                        if (e - p < 5) return fail("bad \\u escape");
                        unsigned v = 0;
                        for (int i = 1; i <= 4; ++i) {
                            const char c = p[i];
                            v = v * 16 + (c >= '0' && c <= '9' ? c - '0' : (c | 32) >= 'a' && (c | 32) <= 'f' ? (c | 32) - 'a' + 10 : 0);
                        }
                        out += v < 128 ? (char)v : '?';
                        p += 4;
                        break;
                    }
                    default: out += *p;
                }
                ++p;
            } else {
                out += *p++;
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JVal &v) {
        if (++depth > 64) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        bool ok = true;
        if (*p == '{') {
            v.kind = JVal::OBJ;
            ++p;
            ws();
            if (p < e && *p == '}') { ++p; --depth; return true; }
            for (;;) {
                ws();
                std::pair<std::string, JVal> kv;
                if (!str(kv.first)) return false;
                ws();
                if (p >= e || *p != ':') return fail("expected ':'");
                ++p;
                if (!value(kv.second)) return false;
                v.obj.push_back(std::move(kv));
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == '}') { ++p; break; }
                return fail("expected ',' or '}'");
            }
        } else if (*p == '[') {
            v.kind = JVal::ARR;
            ++p;
            ws();
            if (p < e && *p == ']') { ++p; --depth; return true; }
            for (;;) {
                JVal x;
                if (!value(x)) return false;
                v.arr.push_back(std::move(x));
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == ']') { ++p; break; }
                return fail("expected ',' or ']'");
            }
        } else if (*p == '"') {
            v.kind = JVal::STR;
            ok = str(v.str);
        } else if (e - p >= 4 && !std::strncmp(p, "true", 4)) {
            v.kind = JVal::BOOL; v.b = true; p += 4;
        } else if (e - p >= 5 && !std::strncmp(p, "false", 5)) {
            v.kind = JVal::BOOL; p += 5;
        } else if (e - p >= 4 && !std::strncmp(p, "null", 4)) {
            p += 4;
        } else {
            const char *q = p;
            bool integer = true;
            if (q < e && (*q == '-' || *q == '+')) ++q;
            while (q < e && ((*q >= '0' && *q <= '9') || *q == '.' || *q == 'e' || *q == 'E' || *q == '-' || *q == '+')) {
                if (*q == '.' || *q == 'e' || *q == 'E') integer = false;
                ++q;
            }
            if (q == p) return fail("unexpected character");
            const std::string tok(p, q);
            v.kind = JVal::NUM;
            v.num = std::strtod(tok.c_str(), nullptr);
            v.is_int = integer;
            if (integer) v.inum = std::strtoll(tok.c_str(), nullptr, 10);
            p = q;
        }
        --depth;
        return ok;
    }
};

// ---- safetensors index -----------------------------------------------------------------
struct STensor {
    std::string dtype;
    std::vector<long long> shape;
    unsigned long long begin = 0, end = 0;
    int file = 0;
};

struct SafeTensors {
    std::vector<std::string> paths;
    std::vector<unsigned long long> data_start, file_size;
    std::map<std::string, STensor> t;

    int open(const char *const *ps, int n) {
        for (int f = 0; f < n; ++f) {
            if (!ps[f]) return set_error(Q35_ERR_INVALID, "safetensors: NULL path");
            FILE *fp = std::fopen(ps[f], "rb");
            if (!fp) return set_error(Q35_ERR_INVALID, std::string("safetensors: cannot open ") + ps[f] + ": " + std::strerror(errno));
            unsigned char hb[8];
            std::fseek(fp, 0, SEEK_END);
            const long long fsz = std::ftell(fp);
            std::fseek(fp, 0, SEEK_SET);
            if (fsz < 8 || std::fread(hb, 1, 8, fp) != 8) {
                std::fclose(fp);
                return set_error(Q35_ERR_INVALID, std::string("safetensors: truncated header in ") + ps[f]);
            }
            unsigned long long hl = 0;
            for (int i = 7; i >= 0; --i) hl = hl << 8 | hb[i];
            if (hl > 100000000ull || 8 + hl > (unsigned long long)fsz) {
                std::fclose(fp);
                return set_error(Q35_ERR_INVALID, std::string("safetensors: bad header length in ") + ps[f]);
            }
            std::string h(hl, '\0');
            const size_t got = std::fread(&h[0], 1, hl, fp);
            std::fclose(fp);
            if (got != hl) return set_error(Q35_ERR_INVALID, std::string("safetensors: short header in ") + ps[f]);
            JParser jp{h.data(), h.data() + h.size()};
            JVal root;
            if (!jp.value(root) || root.kind != JVal::OBJ)
                return set_error(Q35_ERR_INVALID, std::string("safetensors: header of ") + ps[f] + ": " + jp.err);
            const unsigned long long data_bytes = (unsigned long long)fsz - 8 - hl;
            for (const auto &kv : root.obj) {
                if (kv.first == "__metadata__") continue;
                const JVal &d = kv.second;
                const JVal *dt = d.get("dtype"), *sh = d.get("shape"), *off = d.get("data_offsets");
                if (!dt || dt->kind != JVal::STR || !sh || sh->kind != JVal::ARR || !off || off->kind != JVal::ARR ||
                    off->arr.size() != 2 || !off->arr[0].is_int || !off->arr[1].is_int)
                    return set_error(Q35_ERR_INVALID, "safetensors: malformed entry " + kv.first);
                STensor s;
                s.dtype = dt->str;
                for (const JVal &x : sh->arr) {
                    if (x.kind != JVal::NUM || !x.is_int || x.inum < 0)
                        return set_error(Q35_ERR_INVALID, "safetensors: bad shape of " + kv.first);
                    s.shape.push_back(x.inum);
                }
                s.begin = (unsigned long long)off->arr[0].inum;
                s.end = (unsigned long long)off->arr[1].inum;
                s.file = f;
                unsigned long long n_el = 1;
                for (long long x : s.shape) n_el *= (unsigned long long)x;
                const int es = elem_size(s.dtype);
                if (s.end < s.begin || s.end > data_bytes || (es && n_el * es != s.end - s.begin))
                    return set_error(Q35_ERR_INVALID, "safetensors: data range of " + kv.first + " does not fit");
                t[kv.first] = s;
            }
            paths.push_back(ps[f]);
            data_start.push_back(8 + hl);
            file_size.push_back((unsigned long long)fsz);
        }
        return Q35_OK;
    }
    static int elem_size(const std::string &d) {
        if (d == "F32" || d == "I32" || d == "U32") return 4;
        if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
        if (d == "I8" || d == "U8" || d == "BOOL") return 1;
        if (d == "F64" || d == "I64" || d == "U64") return 8;
        return 0;
    }
    const STensor *find(const std::string &k) const {
        auto it = t.find(k);
        return it == t.end() ? nullptr : &it->second;
    }
    int read_raw(const STensor &s, void *dst) const {
        FILE *fp = std::fopen(paths[s.file].c_str(), "rb");
        if (!fp) return set_error(Q35_ERR_INVALID, "safetensors: cannot reopen " + paths[s.file]);
        const unsigned long long off = data_start[s.file] + s.begin, n = s.end - s.begin;
        int st = Q35_OK;
        if (fseeko(fp, (off_t)off, SEEK_SET) != 0 || std::fread(dst, 1, n, fp) != n)
            st = set_error(Q35_ERR_INVALID, "safetensors: short read in " + paths[s.file]);
        std::fclose(fp);
        return st;
    }
};

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1Fu) {
        bits = sign | 0x7F800000u | (man << 13);            // inf / nan
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);   // normal
    } else if (man == 0) {
        bits = sign;                                        // zero
    } else {                                                // subnormal: normalise
        int e = -1;
        do { man <<= 1; ++e; } while (!(man & 0x400u));
        bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// a floating-point tensor of n elements as fp32
int read_float(const SafeTensors &st, const std::string &key, size_t n, std::vector<float> &out) {
    const STensor *s = st.find(key);
    if (!s) return set_error(Q35_ERR_INVALID, "safetensors: missing tensor " + key);
    size_t ne = 1;
    for (long long x : s->shape) ne *= (size_t)x;
    if (ne != n) return set_error(Q35_ERR_INVALID, "safetensors: " + key + " has the wrong size");
    out.resize(n);
    if (s->dtype == "F32") return st.read_raw(*s, out.data());
    if (s->dtype != "F16" && s->dtype != "BF16")
        return set_error(Q35_ERR_INVALID, "safetensors: " + key + " is " + s->dtype + ", not a float type");
    std::vector<uint16_t> h(n);
    int rc = st.read_raw(*s, h.data());
    if (rc) return rc;
    if (s->dtype == "F16") {
        for (size_t i = 0; i < n; ++i) out[i] = half_to_float(h[i]);
    } else {
        for (size_t i = 0; i < n; ++i) {
            const uint32_t b = (uint32_t)h[i] << 16;
            std::memcpy(&out[i], &b, 4);
        }
    }
    return Q35_OK;
}

// key.weight_q [K/2][N] int8 (row-major) -> W_Q(K/2, N) column-major; scales, offsets [N]
int read_q35(const SafeTensors &st, const std::string &key, int K, int N, std::vector<int8_t> &wq,
             std::vector<float> &sc, std::vector<float> &of) {
    const STensor *s = st.find(key + ".weight_q");
    if (!s) return set_error(Q35_ERR_INVALID, "safetensors: missing tensor " + key + ".weight_q");
    if (s->dtype != "I8" && s->dtype != "U8") return set_error(Q35_ERR_INVALID, "safetensors: " + key + ".weight_q is not int8");
    if (s->shape.size() != 2 || s->shape[0] != K / 2 || s->shape[1] != N)
        return set_error(Q35_ERR_INVALID, "safetensors: " + key + ".weight_q shape is not [" + std::to_string(K / 2) +
                                              "][" + std::to_string(N) + "]");
    std::vector<int8_t> rm((size_t)(K / 2) * N);
    int rc = st.read_raw(*s, rm.data());
    if (rc) return rc;
    wq.resize(rm.size());
    const size_t P = (size_t)K / 2;
    for (size_t p0 = 0; p0 < P; p0 += 64)          // blocked transpose
        for (size_t j0 = 0; j0 < (size_t)N; j0 += 64)
            for (size_t p = p0; p < std::min(P, p0 + 64); ++p)
                for (size_t j = j0; j < std::min((size_t)N, j0 + 64); ++j) wq[p + P * j] = rm[p * N + j];
    rc = read_float(st, key + ".scales", (size_t)N, sc);
    if (!rc) rc = read_float(st, key + ".offsets", (size_t)N, of);
    return rc;
}

// a [rows][cols] matrix kept as floats, or quantized as key.weight_q/.scales/.offsets over
// K = rows (expanded: code * scale + zero_point); out row-major [rows][cols]
int read_dense_or_q35(const SafeTensors &st, const std::string &key, int rows, int cols, std::vector<float> &out) {
    if (st.find(key)) return read_float(st, key, (size_t)rows * cols, out);
    if (rows % 2) return set_error(Q35_ERR_INVALID, "safetensors: missing tensor " + key);
    std::vector<int8_t> wq;
    std::vector<float> sc, of;
    int rc = read_q35(st, key, rows, cols, wq, sc, of);
    if (rc) return rc;
    out.resize((size_t)rows * cols);
    const size_t P = (size_t)rows / 2;
    for (size_t j = 0; j < (size_t)cols; ++j)
        for (size_t p = 0; p < P; ++p) {
            const int raw = wq[p + P * j] & 0x7F;
            const int n1 = (raw >> 3) >= 8 ? (raw >> 3) - 16 : (raw >> 3);
            const int n2 = (raw & 7) >= 4 ? (raw & 7) - 8 : (raw & 7);
            out[(2 * p) * cols + j] = (float)n1 * sc[j] + of[j];
            out[(2 * p + 1) * cols + j] = (float)n2 * sc[j] + of[j];
        }
    return Q35_OK;
}

}  // namespace

extern "C" {

int q35_model_load_layer_file(q35_model m, int32_t layer, const char *path) {
    if (!m || !path) return set_error(Q35_ERR_INVALID, "NULL argument");
    const q35_model_config &c = model_config(m);
    if (c.wformat != Q35_FMT_INT4)
        return set_error(Q35_ERR_INVALID, "layer file: the stream-binary layer file holds INT4 weights (scales only)");
    if (layer < 0 || layer >= c.n_layers) return set_error(Q35_ERR_INVALID, "layer index out of range");
    const long long hid = c.hidden, QN = (long long)c.n_heads * c.head_dim, KN = (long long)c.n_kv_heads * c.head_dim,
                    F = c.ffn;
    const long long shapes[7][2] = {{hid, QN}, {hid, KN}, {hid, KN}, {QN, hid}, {hid, F}, {hid, F}, {F, hid}};
    long long need = 0;
    for (auto &kn : shapes) need += kn[0] / 2 * kn[1] + 4 * kn[1];
    FILE *fp = std::fopen(path, "rb");
    if (!fp) return set_error(Q35_ERR_INVALID, std::string("layer file: cannot open ") + path + ": " + std::strerror(errno));
    std::fseek(fp, 0, SEEK_END);
    const long long fsz = std::ftell(fp);
    std::fseek(fp, 0, SEEK_SET);
    const bool norms = fsz == need + 8 * hid;
    if (fsz != need && !norms) {
        std::fclose(fp);
        return set_error(Q35_ERR_INVALID, std::string("layer file: ") + path + " holds " + std::to_string(fsz) +
                                              " bytes; this model's layer needs " + std::to_string(need) + " (or " +
                                              std::to_string(need + 8 * hid) + " with the two norms)");
    }
    std::vector<int8_t> w[7];
    std::vector<float> s[7], an, fn;
    int st = Q35_OK;
    for (int i = 0; i < 7 && !st; ++i) {
        w[i].resize((size_t)(shapes[i][0] / 2 * shapes[i][1]));
        s[i].resize((size_t)shapes[i][1]);
        if (std::fread(w[i].data(), 1, w[i].size(), fp) != w[i].size() ||
            std::fread(s[i].data(), 4, s[i].size(), fp) != s[i].size())
            st = set_error(Q35_ERR_INVALID, std::string("layer file: short read in ") + path);
    }
    if (!st && norms) {
        an.resize((size_t)hid);
        fn.resize((size_t)hid);
        if (std::fread(an.data(), 4, an.size(), fp) != an.size() || std::fread(fn.data(), 4, fn.size(), fp) != fn.size())
            st = set_error(Q35_ERR_INVALID, std::string("layer file: short read in ") + path);
    }
    std::fclose(fp);
    if (st) return st;
    q35_layer_weights lw{};
    lw.wq = w[0].data(); lw.wk = w[1].data(); lw.wv = w[2].data(); lw.wo = w[3].data();
    lw.wg = w[4].data(); lw.wu = w[5].data(); lw.wd = w[6].data();
    lw.sq = s[0].data(); lw.sk = s[1].data(); lw.sv = s[2].data(); lw.so = s[3].data();
    lw.sg = s[4].data(); lw.su = s[5].data(); lw.sd = s[6].data();
    lw.attn_norm = norms ? an.data() : nullptr;
    lw.ffn_norm = norms ? fn.data() : nullptr;
    return q35_model_set_layer(m, layer, &lw);
}

int q35_model_load_safetensors(q35_model m, const char *const *paths, int32_t n_paths) {
    if (!m || !paths || n_paths < 1) return set_error(Q35_ERR_INVALID, "NULL argument");
    const q35_model_config &c = model_config(m);
    if (c.wformat != Q35_FMT_3P5BIT)
        return set_error(Q35_ERR_INVALID, "safetensors: the 3.5-bit file needs a 3.5-bit model");
    SafeTensors st;
    int rc = st.open(paths, n_paths);
    if (rc) return rc;
    const int hid = c.hidden, QN = c.n_heads * c.head_dim, KN = c.n_kv_heads * c.head_dim, F = c.ffn, V = c.vocab;
    static const char *names[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                   "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"};
    const int shapes[7][2] = {{hid, QN}, {hid, KN}, {hid, KN}, {QN, hid}, {hid, F}, {hid, F}, {F, hid}};
    for (int l = 0; l < c.n_layers; ++l) {
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        std::vector<int8_t> w[7];
        std::vector<float> s[7], o[7], an, fn;
        for (int i = 0; i < 7; ++i) {
            rc = read_q35(st, pre + names[i] + ".weight", shapes[i][0], shapes[i][1], w[i], s[i], o[i]);
            if (rc) return rc;
        }
        rc = read_float(st, pre + "input_layernorm.weight", (size_t)hid, an);
        if (!rc) rc = read_float(st, pre + "post_attention_layernorm.weight", (size_t)hid, fn);
        if (rc) return rc;
        q35_layer_weights lw{};
        lw.wq = w[0].data(); lw.wk = w[1].data(); lw.wv = w[2].data(); lw.wo = w[3].data();
        lw.wg = w[4].data(); lw.wu = w[5].data(); lw.wd = w[6].data();
        lw.sq = s[0].data(); lw.sk = s[1].data(); lw.sv = s[2].data(); lw.so = s[3].data();
        lw.sg = s[4].data(); lw.su = s[5].data(); lw.sd = s[6].data();
        lw.oq = o[0].data(); lw.ok = o[1].data(); lw.ov = o[2].data(); lw.oo = o[3].data();
        lw.og = o[4].data(); lw.ou = o[5].data(); lw.od = o[6].data();
        lw.attn_norm = an.data();
        lw.ffn_norm = fn.data();
        rc = q35_model_set_layer(m, l, &lw);
        if (rc) return rc;
    }
    std::vector<float> emb, head, fnorm;
    rc = read_dense_or_q35(st, "model.embed_tokens.weight", V, hid, emb);
    if (!rc) rc = read_float(st, "model.norm.weight", (size_t)hid, fnorm);
    if (!rc) rc = read_dense_or_q35(st, "lm_head.weight", V, hid, head);
    if (rc) return rc;
    return model_set_embeddings_rm(m, emb.data(), fnorm.data(), head.data());
}

}  // extern "C"
