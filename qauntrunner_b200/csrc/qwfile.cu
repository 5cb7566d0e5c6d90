// qwfile.cu -- QuantRunner .qw weight files as a source of MoE layers.
//
// The .qw format (src/QuantRunner.Core/Memory/ModelStore.cs:44-126): bytes
// "QWR1", an int32 header length, a UTF-8 JSON header
//   {"config": {...ModelConfig...}, "tensors": [{"name", "dims", "format",
//    "offset", "size"}, ...], "data_offset"?: N}
// and the tensor data from data_offset (or 8 + header length) rounded up to
// 64 bytes; tensor offsets are relative to that start.  Names are the
// canonical ones of NameMapper.cs:7-12 (l{i}.ffn_norm, l{i}.router,
// l{i}.router_bias, l{i}.e{j}.w_gate / w_up / w_down, l{i}.sw_*).
//
// qrm_qw_layer_desc reads a layer's description from the header (no GPU
// work); qrm_load_qw maps the file read-only and uploads one layer's MoE
// tensors by name through the layer's own upload entry points, so expert
// blocks go to HBM as they are stored (no requantisation).  Host code only.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "qrmoe.h"

extern "C" int qrm_set_error(int code, const char* msg);   // qrmoe.cu

namespace {

int qw_fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return qrm_set_error(code, buf);
}

// ---------------------------------------------------------------- JSON
// A small DOM for the header: objects keep their key order, numbers keep
// their text (64-bit offsets parse exactly as integers).
struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    std::string text;   // number text or string value
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal* get(const char* key) const {
        if (kind != Obj) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    bool as_i64(long long* v) const {
        if (kind != Num) return false;
        char* end = nullptr;
        errno = 0;
        long long x = strtoll(text.c_str(), &end, 10);
        if (errno || !end || *end) {
            // integral values written in floating form (e.g. 4.096E+03)
            double dv = strtod(text.c_str(), &end);
            if (!end || *end || dv != std::floor(dv) || std::fabs(dv) > 9.0e15) return false;
            x = (long long)dv;
        }
        *v = x;
        return true;
    }
    bool as_f64(double* v) const {
        if (kind != Num) return false;
        char* end = nullptr;
        *v = strtod(text.c_str(), &end);
        return end && !*end;
    }
};

struct JParser {
    const char* p;
    const char* e;
    std::string err;

    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool lit(const char* s) {
        const size_t n = strlen(s);
        if ((size_t)(e - p) < n || memcmp(p, s, n)) return false;
        p += n;
        return true;
    }
    static void put_utf8(std::string& o, unsigned cp) {
        if (cp < 0x80) {
            o += (char)cp;
        } else if (cp < 0x800) {
            o += (char)(0xC0 | (cp >> 6));
            o += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            o += (char)(0xE0 | (cp >> 12));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        } else {
            o += (char)(0xF0 | (cp >> 18));
            o += (char)(0x80 | ((cp >> 12) & 0x3F));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(unsigned* v) {
        if (e - p < 4) return fail("short \\u escape");
        unsigned x = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p++;
            x <<= 4;
            if (c >= '0' && c <= '9') x |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') x |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') x |= (unsigned)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        *v = x;
        return true;
    }
    bool str(std::string& o) {
        if (p >= e || *p != '"') return fail("expected a string");
        p++;
        while (p < e && *p != '"') {
            if (*p != '\\') {
                o += *p++;
                continue;
            }
            if (++p >= e) return fail("bad escape");
            const char c = *p++;
            switch (c) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                        p += 2;
                        unsigned lo;
                        if (!hex4(&lo)) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    put_utf8(o, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= e) return fail("unterminated string");
        p++;
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        const char c = *p;
        if (c == '{') {
            v.kind = JVal::Obj;
            p++;
            ws();
            if (p < e && *p == '}') { p++; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= e || *p != ':') return fail("expected ':'");
                p++;
                v.obj.emplace_back(std::move(k), JVal());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p < e && *p == ',') { p++; continue; }
                if (p < e && *p == '}') { p++; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = JVal::Arr;
            p++;
            ws();
            if (p < e && *p == ']') { p++; return true; }
            for (;;) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p < e && *p == ',') { p++; continue; }
                if (p < e && *p == ']') { p++; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = JVal::Str;
            return str(v.text);
        }
        if (lit("true")) { v.kind = JVal::Bool; v.b = true; return true; }
        if (lit("false")) { v.kind = JVal::Bool; v.b = false; return true; }
        if (lit("null")) { v.kind = JVal::Null; return true; }
        const char* s = p;
        if (p < e && (*p == '-' || *p == '+')) p++;
        while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) p++;
        if (p == s) return fail("unexpected character");
        v.kind = JVal::Num;
        v.text.assign(s, p);
        return true;
    }
};

// ---------------------------------------------------------------- file
struct Tensor {
    std::vector<long long> dims;
    int fmt = -1;
    long long offset = 0, size = 0;
    long long numel() const {
        long long n = 1;
        for (long long x : dims) n *= x;
        return n;
    }
};

struct QwFile {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t bytes = 0;
    long long data = 0;
    JVal root;
    std::map<std::string, Tensor> tensors;
    ~QwFile() {
        if (base) munmap(const_cast<uint8_t*>(base), bytes);
        if (fd >= 0) close(fd);
    }
    const Tensor* find(const std::string& n) const {
        auto it = tensors.find(n);
        return it == tensors.end() ? nullptr : &it->second;
    }
    const uint8_t* ptr(const Tensor& t) const { return base + data + t.offset; }
};

// Opens and maps the file, checks magic and header (ModelStore.Open,
// ModelStore.cs:85-126) and every tensor's extent.
int qw_open(const char* path, QwFile& f) {
    if (!path) return qw_fail(QRM_E_INVALID, "path is NULL");
    f.fd = open(path, O_RDONLY | O_CLOEXEC);
    if (f.fd < 0) return qw_fail(QRM_E_INVALID, "%s: cannot open (%s)", path, strerror(errno));
    struct stat st;
    if (fstat(f.fd, &st) != 0) return qw_fail(QRM_E_INVALID, "%s: cannot stat", path);
    f.bytes = (size_t)st.st_size;
    if (f.bytes < 8) return qw_fail(QRM_E_INVALID, "%s: not a QuantRunner .qw file", path);
    void* m = mmap(nullptr, f.bytes, PROT_READ, MAP_PRIVATE, f.fd, 0);
    if (m == MAP_FAILED) return qw_fail(QRM_E_INVALID, "%s: mmap failed (%s)", path, strerror(errno));
    f.base = static_cast<const uint8_t*>(m);
    if (memcmp(f.base, "QWR1", 4) != 0) return qw_fail(QRM_E_INVALID, "%s: not a QuantRunner .qw file", path);
    int32_t hlen;
    memcpy(&hlen, f.base + 4, 4);
    if (hlen < 2 || (size_t)hlen > f.bytes - 8) return qw_fail(QRM_E_INVALID, "%s: corrupt header length %d", path, hlen);
    JParser jp{reinterpret_cast<const char*>(f.base + 8), reinterpret_cast<const char*>(f.base + 8 + hlen), {}};
    if (!jp.value(f.root, 0) || f.root.kind != JVal::Obj)
        return qw_fail(QRM_E_INVALID, "%s: header is not valid JSON (%s)", path, jp.err.c_str());
    long long ds = 8LL + hlen;
    if (const JVal* d = f.root.get("data_offset")) {
        long long v;
        if (d->as_i64(&v)) ds = v;
    }
    ds = (ds + 63) & ~63LL;
    if (ds < 8LL + hlen) return qw_fail(QRM_E_INVALID, "%s: corrupt header (data_offset %lld < header end %lld)", path, ds,
                                        8LL + hlen);
    f.data = ds;
    const JVal* ts = f.root.get("tensors");
    if (!ts || ts->kind != JVal::Arr) return qw_fail(QRM_E_INVALID, "%s: header has no tensor list", path);
    for (const JVal& te : ts->arr) {
        const JVal* n = te.get("name");
        const JVal* dims = te.get("dims");
        const JVal* fm = te.get("format");
        const JVal* off = te.get("offset");
        const JVal* sz = te.get("size");
        Tensor t;
        long long v;
        if (!n || n->kind != JVal::Str || !dims || dims->kind != JVal::Arr || !fm || !fm->as_i64(&v) || !off || !sz)
            return qw_fail(QRM_E_INVALID, "%s: malformed tensor entry", path);
        t.fmt = (int)v;
        for (const JVal& x : dims->arr) {
            if (!x.as_i64(&v) || v < 0) return qw_fail(QRM_E_INVALID, "%s: %s: bad dims", path, n->text.c_str());
            t.dims.push_back(v);
        }
        if (!off->as_i64(&t.offset) || !sz->as_i64(&t.size) || t.offset < 0 || t.size < 0 ||
            (unsigned long long)f.data + t.offset + t.size > f.bytes)
            return qw_fail(QRM_E_INVALID, "%s: %s lies outside the file", path, n->text.c_str());
        f.tensors[n->text] = t;
    }
    return QRM_OK;
}

double cfg_num(const JVal* cfg, const char* key, double dflt) {
    const JVal* v = cfg ? cfg->get(key) : nullptr;
    double x;
    if (v && v->kind == JVal::Bool) return v->b ? 1.0 : 0.0;
    if (v && v->as_f64(&x)) return x;
    return dflt;
}

std::string lname(int layer, const char* rest) { return "l" + std::to_string(layer) + "." + rest; }
std::string ename(int layer, int e, const char* w) {
    return "l" + std::to_string(layer) + ".e" + std::to_string(e) + "." + w;
}

// exact binary16 -> binary32 (Dtypes.cs:76-103 semantics: normals,
// subnormals, infinities and NaNs)
float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        const float v = (float)man * 5.9604644775390625e-8f;   // man * 2^-24, exact
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// a float tensor (F32, F16 or BF16) of n elements widened to f32 (exact)
int widen(const QwFile& f, const std::string& name, const Tensor& t, long long n, std::vector<float>& out) {
    if (t.numel() != n) return qw_fail(QRM_E_SIZE, "%s has %lld elements, expected %lld", name.c_str(), t.numel(), n);
    const int es = t.fmt == QRM_F32 ? 4 : (t.fmt == QRM_F16 || t.fmt == QRM_BF16) ? 2 : 0;
    if (!es) return qw_fail(QRM_E_FORMAT, "%s: format %d (the layer takes F32, F16 or BF16 here)", name.c_str(), t.fmt);
    if (t.size != n * es) return qw_fail(QRM_E_SIZE, "%s: %lld bytes for %lld elements", name.c_str(), t.size, n);
    out.resize((size_t)n);
    const uint8_t* p = f.ptr(t);
    for (long long i = 0; i < n; i++) {
        if (t.fmt == QRM_F32) {
            memcpy(&out[i], p + 4 * i, 4);
        } else {
            uint16_t h;
            memcpy(&h, p + 2 * i, 2);
            if (t.fmt == QRM_F16) {
                out[i] = half_to_float(h);
            } else {
                const uint32_t b = (uint32_t)h << 16;
                memcpy(&out[i], &b, 4);
            }
        }
    }
    return QRM_OK;
}

}  // namespace

extern "C" int qrm_qw_layer_desc(const char* path, int layer_index, int device, int max_tokens, qrm_layer_desc* out) {
    if (!out) return qw_fail(QRM_E_INVALID, "out is NULL");
    QwFile f;
    int rc = qw_open(path, f);
    if (rc) return rc;
    const JVal* cfg = f.root.get("config");
    if (!cfg || cfg->kind != JVal::Obj) return qw_fail(QRM_E_INVALID, "%s: header has no config", path);
    const int L = layer_index;
    if (!f.find(lname(L, "router")))
        return qw_fail(QRM_E_STATE, "%s: layer %d has no router (a dense FFN layer, StreamingEngine.cs:633-637)", path, L);
    qrm_layer_desc d{};
    d.d_model = (int)cfg_num(cfg, "dim", 0);
    d.n_experts = (int)cfg_num(cfg, "n_experts", 0);
    d.n_active = (int)cfg_num(cfg, "n_active", 0);
    const double ef = cfg_num(cfg, "expert_ffn", -1);
    d.expert_ffn = (int)(ef > 0 ? ef : cfg_num(cfg, "ffn", 0));   // ModelConfig.EffectiveExpertFfn
    d.moe_sigmoid = cfg_num(cfg, "moe_sigmoid", 0) != 0 ? 1 : 0;
    d.routed_scale = (float)cfg_num(cfg, "routed_scale", 1.0);
    d.n_shared = (int)cfg_num(cfg, "n_shared", 0);
    d.swiglu_limit = (float)cfg_num(cfg, "swiglu_limit", 0.0);
    d.rms_eps = (float)cfg_num(cfg, "rms_eps", 1e-5);
    const Tensor* g = f.find(ename(L, 0, "w_gate"));
    const Tensor* u = f.find(ename(L, 0, "w_up"));
    const Tensor* dn = f.find(ename(L, 0, "w_down"));
    if (!g || !u || !dn) return qw_fail(QRM_E_STATE, "%s: layer %d has no expert 0 matrices", path, L);
    d.fmt_gate = g->fmt;
    d.fmt_up = u->fmt;
    d.fmt_down = dn->fmt;
    // the shared expert runs only when its tensors exist (StreamingEngine.cs:779)
    const Tensor* sg = f.find(lname(L, "sw_gate"));
    const Tensor* su = f.find(lname(L, "sw_up"));
    const Tensor* sd = f.find(lname(L, "sw_down"));
    if (d.n_shared > 0 && d.moe_sigmoid && sg && su && sd) {
        d.fmt_sh_gate = sg->fmt;
        d.fmt_sh_up = su->fmt;
        d.fmt_sh_down = sd->fmt;
    } else {
        d.n_shared = 0;
        d.fmt_sh_gate = d.fmt_gate;
        d.fmt_sh_up = d.fmt_up;
        d.fmt_sh_down = d.fmt_down;
    }
    d.device = device;
    d.max_tokens = max_tokens;
    *out = d;
    return QRM_OK;
}

extern "C" int qrm_load_qw(qrm_layer* layer, const char* path, int layer_index) {
    if (!layer) return qw_fail(QRM_E_INVALID, "NULL layer");
    QwFile f;
    int rc = qw_open(path, f);
    if (rc) return rc;
    qrm_layer_desc d;
    rc = qrm_layer_get_desc(layer, &d);
    if (rc) return rc;
    const int L = layer_index;
    std::vector<float> buf, bias;
    // RMSNorm weights (optional: a caller that normalises itself needs none)
    if (const Tensor* t = f.find(lname(L, "ffn_norm"))) {
        if ((rc = widen(f, lname(L, "ffn_norm"), *t, d.d_model, buf))) return rc;
        if ((rc = qrm_upload_norm(layer, buf.data()))) return rc;
    }
    // router [E x d] and GLM router bias [E]
    const Tensor* rt = f.find(lname(L, "router"));
    if (!rt) return qw_fail(QRM_E_STATE, "%s: tensor 'l%d.router' not found", path, L);
    if (rt->dims.size() != 2 || rt->dims[0] != d.n_experts || rt->dims[1] != d.d_model)
        return qw_fail(QRM_E_INVALID, "%s: l%d.router is not [%d x %d]", path, L, d.n_experts, d.d_model);
    if ((rc = widen(f, lname(L, "router"), *rt, (long long)d.n_experts * d.d_model, buf))) return rc;
    const Tensor* bt = f.find(lname(L, "router_bias"));
    if (bt && d.moe_sigmoid) {
        if ((rc = widen(f, lname(L, "router_bias"), *bt, d.n_experts, bias))) return rc;
    }
    if ((rc = qrm_upload_router(layer, buf.data(), bias.empty() ? nullptr : bias.data()))) return rc;
    std::vector<float>().swap(buf);
    // expert matrices of the experts this layer holds, as stored
    int first = 0, count = d.n_experts;
    if ((rc = qrm_expert_range(layer, &first, &count))) return rc;
    static const char* kW[3] = {"w_gate", "w_up", "w_down"};
    for (int e = first; e < first + count; e++) {
        for (int w = 0; w < 3; w++) {
            const std::string n = ename(L, e, kW[w]);
            const Tensor* t = f.find(n);
            if (!t) return qw_fail(QRM_E_STATE, "%s: tensor '%s' not found", path, n.c_str());
            const long long rows = w == 2 ? d.d_model : d.expert_ffn, cols = w == 2 ? d.expert_ffn : d.d_model;
            if (t->dims.size() != 2 || t->dims[0] != rows || t->dims[1] != cols)
                return qw_fail(QRM_E_INVALID, "%s: %s is not [%lld x %lld]", path, n.c_str(), rows, cols);
            if ((rc = qrm_upload_expert(layer, e, w, t->fmt, f.ptr(*t), (size_t)t->size))) return rc;
        }
    }
    if (d.moe_sigmoid && d.n_shared > 0) {
        static const char* kS[3] = {"sw_gate", "sw_up", "sw_down"};
        for (int w = 0; w < 3; w++) {
            const std::string n = lname(L, kS[w]);
            const Tensor* t = f.find(n);
            if (!t) return qw_fail(QRM_E_STATE, "%s: tensor '%s' not found", path, n.c_str());
            const long long rows = w == 2 ? d.d_model : d.expert_ffn, cols = w == 2 ? d.expert_ffn : d.d_model;
            if (t->dims.size() != 2 || t->dims[0] != rows || t->dims[1] != cols)
                return qw_fail(QRM_E_INVALID, "%s: %s is not [%lld x %lld]", path, n.c_str(), rows, cols);
            if ((rc = qrm_upload_expert(layer, QRM_SHARED_EXPERT, w, t->fmt, f.ptr(*t), (size_t)t->size))) return rc;
        }
    }
    return QRM_OK;
}
