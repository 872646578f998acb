// poolfile.cu -- the converter's pool layout file: the JSON written next to
// a packed expert pool (tools/convert-ds4f.py:1321-1393) and read by the
// engine with ds4f_pool_layout_load (src/moe.c:51-160). Host code only.
//
// The packed file is [u64 expert_nbytes][u64 n_layers][u64 n_experts] then
// one fixed-size slot per expert, layer-major. Within a slot the converter
// writes each tensor's values then its scales, in the order of its sorted
// tensor names (tools/convert-ds4f.py:1242), so a Qwen slot holds down_proj,
// gate_proj, up_proj; the engine instead reads the tensor entries as gate,
// up, down (src/moe.c:598-605). This reader places every tensor by its name
// when the entry has one ("n"), else by its position among the expert's
// entries (the engine's rule), and copies it to this library's slot layout
// (gate, up, down; values then scales each).
//
// Refusals follow the engine's: missing top-level keys, a layer/expert count
// other than the model's, a tensor outside its slot (src/moe.c:64-82,
// :139-148); entries without the per-tensor keys, or with a layer or expert
// out of range, are skipped as there (:97-101). Added, because this path
// computes with the bytes rather than trusting them: a tensor whose shape or
// byte counts differ from the model's, a role given twice, or an expert
// without all three roles.
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <string>
#include <unistd.h>
#include <vector>

#include "common.cuh"
#include "matvec.cuh"
#include "model.cuh"
#include "../../include/ds4f/gpu_cuda.h"

namespace ds4f {
namespace {

// ---- a small JSON reader (RFC 8259 values; numbers kept as int64 when
// ---- written without fraction or exponent) -------------------------------
struct JVal {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    bool is_int = false, b = false;
    int64_t i = 0;
    double d = 0;
    std::string s;
    std::vector<JVal> a;
    std::vector<std::pair<std::string, JVal>> o;

    const JVal *get(const char *key) const {
        if (kind != kObj) return nullptr;
        for (const auto &kv : o)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JReader {
  public:
    JReader(const char *p, size_t n) : p_(p), b_(p), e_(p + n) {}
    bool parse(JVal &root) {
        ws();
        if (!value(root, 0)) return false;
        ws();
        if (p_ != e_) return fail("trailing characters");
        return true;
    }
    std::string error() const {
        char buf[160];
        snprintf(buf, sizeof buf, "%s at byte %lld", err_.c_str(), (long long)(at_ - b_));
        return buf;
    }

  private:
    const char *p_, *b_, *e_, *at_ = nullptr;
    std::string err_;

    bool fail(const char *m) {
        if (err_.empty()) { err_ = m; at_ = p_; }
        return false;
    }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) p_++;
    }
    bool lit(const char *w) {
        size_t n = strlen(w);
        if ((size_t)(e_ - p_) < n || memcmp(p_, w, n)) return fail("bad literal");
        p_ += n;
        return true;
    }
    static void utf8(std::string &s, uint32_t c) {
        if (c < 0x80) s += (char)c;
        else if (c < 0x800) { s += (char)(0xC0 | (c >> 6)); s += (char)(0x80 | (c & 63)); }
        else if (c < 0x10000) {
            s += (char)(0xE0 | (c >> 12)); s += (char)(0x80 | ((c >> 6) & 63)); s += (char)(0x80 | (c & 63));
        } else {
            s += (char)(0xF0 | (c >> 18)); s += (char)(0x80 | ((c >> 12) & 63));
            s += (char)(0x80 | ((c >> 6) & 63)); s += (char)(0x80 | (c & 63));
        }
    }
    bool hex4(uint32_t &c) {
        if (e_ - p_ < 4) return fail("short \\u escape");
        c = 0;
        for (int k = 0; k < 4; k++, p_++) {
            char h = *p_;
            c <<= 4;
            if (h >= '0' && h <= '9') c |= (uint32_t)(h - '0');
            else if (h >= 'a' && h <= 'f') c |= (uint32_t)(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') c |= (uint32_t)(h - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool str(std::string &s) {
        if (p_ >= e_ || *p_ != '"') return fail("expected a string");
        p_++;
        while (true) {
            if (p_ >= e_) return fail("unterminated string");
            unsigned char c = (unsigned char)*p_++;
            if (c == '"') return true;
            if (c < 0x20) return fail("control character in string");
            if (c != '\\') { s += (char)c; continue; }
            if (p_ >= e_) return fail("unterminated escape");
            char x = *p_++;
            switch (x) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    uint32_t c1;
                    if (!hex4(c1)) return false;
                    if (c1 >= 0xD800 && c1 < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        uint32_t c2;
                        if (!hex4(c2)) return false;
                        if (c2 < 0xDC00 || c2 > 0xDFFF) return fail("bad surrogate pair");
                        c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                    }
                    utf8(s, c1);
                    break;
                }
                default: return fail("bad escape");
            }
        }
    }
    bool num(JVal &v) {
        const char *q = p_;
        if (q < e_ && *q == '-') q++;
        if (q >= e_ || *q < '0' || *q > '9') return fail("bad number");
        if (*q == '0' && q + 1 < e_ && q[1] >= '0' && q[1] <= '9') return fail("leading zero");
        while (q < e_ && *q >= '0' && *q <= '9') q++;
        bool frac = false;
        if (q < e_ && *q == '.') {
            frac = true; q++;
            if (q >= e_ || *q < '0' || *q > '9') return fail("bad fraction");
            while (q < e_ && *q >= '0' && *q <= '9') q++;
        }
        if (q < e_ && (*q == 'e' || *q == 'E')) {
            frac = true; q++;
            if (q < e_ && (*q == '+' || *q == '-')) q++;
            if (q >= e_ || *q < '0' || *q > '9') return fail("bad exponent");
            while (q < e_ && *q >= '0' && *q <= '9') q++;
        }
        std::string t(p_, q);
        v.kind = JVal::kNum;
        v.d = strtod(t.c_str(), nullptr);
        if (!frac) {
            errno = 0;
            long long ll = strtoll(t.c_str(), nullptr, 10);
            if (errno == ERANGE) return fail("integer out of range");
            v.is_int = true;
            v.i = ll;
        }
        p_ = q;
        return true;
    }
    bool value(JVal &v, int depth) {
        if (depth > 64) return fail("nesting deeper than 64");
        ws();
        if (p_ >= e_) return fail("unexpected end");
        switch (*p_) {
            case '{': {
                p_++;
                v.kind = JVal::kObj;
                ws();
                if (p_ < e_ && *p_ == '}') { p_++; return true; }
                while (true) {
                    ws();
                    std::string k;
                    if (!str(k)) return false;
                    ws();
                    if (p_ >= e_ || *p_ != ':') return fail("expected ':'");
                    p_++;
                    v.o.emplace_back(std::move(k), JVal());
                    if (!value(v.o.back().second, depth + 1)) return false;
                    ws();
                    if (p_ < e_ && *p_ == ',') { p_++; continue; }
                    if (p_ < e_ && *p_ == '}') { p_++; return true; }
                    return fail("expected ',' or '}'");
                }
            }
            case '[': {
                p_++;
                v.kind = JVal::kArr;
                ws();
                if (p_ < e_ && *p_ == ']') { p_++; return true; }
                while (true) {
                    v.a.emplace_back();
                    if (!value(v.a.back(), depth + 1)) return false;
                    ws();
                    if (p_ < e_ && *p_ == ',') { p_++; continue; }
                    if (p_ < e_ && *p_ == ']') { p_++; return true; }
                    return fail("expected ',' or ']'");
                }
            }
            case '"': v.kind = JVal::kStr; return str(v.s);
            case 't': v.kind = JVal::kBool; v.b = true; return lit("true");
            case 'f': v.kind = JVal::kBool; v.b = false; return lit("false");
            case 'n': v.kind = JVal::kNull; return lit("null");
            default: return num(v);
        }
    }
};

bool get_int(const JVal &o, const char *k, int64_t *out) {
    const JVal *v = o.get(k);
    if (!v || v->kind != JVal::kNum || !v->is_int) return false;
    *out = v->i;
    return true;
}

bool ends_with(const std::string &s, const char *suf) {
    size_t n = strlen(suf);
    return s.size() >= n && !s.compare(s.size() - n, n, suf);
}

const char *kRoleName[3] = {"gate_proj", "up_proj", "down_proj"};

}  // namespace

// Absolute file offsets of every expert's six pieces -- values then scales
// of gate, up, down -- from the layout file, checked against the model
// shape (fmt, H, M, L, E). off is [L*E*6]; *nbytes receives expert_nbytes.
int pool_plan(const char *json_path, int fmt, int H, int M, int L, int E, std::vector<int64_t> &off,
              int64_t *nbytes) {
    SlotLayout sl;
    DS4F_REQUIRE(L > 0 && E > 0, "pool layout: %d layers x %d experts", L, E);
    if (slot_layout(fmt, H, M, &sl)) return -1;
    const int64_t vb = sl.rel_s[0] - sl.rel_v[0], sb = sl.rel_v[1] - sl.rel_s[0];
    FILE *f = fopen(json_path, "rb");
    DS4F_REQUIRE(f, "pool layout: cannot read %s", json_path);
    std::string buf;
    {
        char tmp[1 << 16];
        size_t n;
        while ((n = fread(tmp, 1, sizeof tmp, f)) > 0) buf.append(tmp, n);
        fclose(f);
    }
    JVal root;
    JReader rd(buf.data(), buf.size());
    DS4F_REQUIRE(rd.parse(root), "pool layout: %s not parseable (%s)", json_path, rd.error().c_str());
    buf.clear();
    buf.shrink_to_fit();
    int64_t nl, ne, nb;
    const JVal *ts = root.get("tensors");
    DS4F_REQUIRE(root.kind == JVal::kObj && get_int(root, "n_layers", &nl) && get_int(root, "n_experts", &ne) &&
                     get_int(root, "expert_nbytes", &nb) && ts && ts->kind == JVal::kArr,
                 "pool layout: %s missing keys (n_layers, n_experts, expert_nbytes, tensors)", json_path);
    DS4F_REQUIRE(nl == L && ne == E, "pool layout: %lldx%lld vs model %dx%d", (long long)nl, (long long)ne, L, E);
    // every slot offset 24 + (L E) nb below must stay inside int64
    DS4F_REQUIRE(nb > 0 && nb <= (INT64_MAX - 24) / ((int64_t)L * E), "pool layout: expert_nbytes %lld",
                 (long long)nb);
    if (const JVal *fm = root.get("format")) {
        const char *want = fmt == DS4F_FMT_FP8 ? "fp8-pool-v1" : "mxfp4-pool-v1";
        DS4F_REQUIRE(fm->kind == JVal::kStr && fm->s == want, "pool layout: format \"%s\", this model reads \"%s\"",
                     fm->kind == JVal::kStr ? fm->s.c_str() : "?", want);
    }
    if (fmt == DS4F_FMT_MXFP4) {
        int64_t bs;
        if (get_int(root, "block_size", &bs))
            DS4F_REQUIRE(bs == 32, "pool layout: MXFP4 block size %lld, 32 expected", (long long)bs);
    }
    off.assign((size_t)L * E * 6, -1);
    std::vector<uint8_t> seen((size_t)L * E, 0);   // roles present, one bit each
    std::vector<uint8_t> count((size_t)L * E, 0);  // entries met
    for (const JVal &t : ts->a) {
        int64_t l, x, vo, so, vn, sn;
        const JVal *shp = t.get("shape");
        if (t.kind != JVal::kObj || !get_int(t, "layer", &l) || !get_int(t, "expert", &x) || !shp ||
            shp->kind != JVal::kArr || !get_int(t, "v_off", &vo) || !get_int(t, "s_off", &so) ||
            !get_int(t, "v_nbytes", &vn) || !get_int(t, "s_nbytes", &sn))
            continue;
        if (l < 0 || l >= L || x < 0 || x >= E) continue;
        const size_t ex = (size_t)l * E + x;
        int role = -1;
        const JVal *nm = t.get("n");
        if (nm && nm->kind == JVal::kStr) {
            for (int r = 0; r < 3; r++) {
                std::string suf = std::string(".") + kRoleName[r] + ".weight";
                if (ends_with(nm->s, suf.c_str())) role = r;
            }
            DS4F_REQUIRE(role >= 0, "pool layout: tensor %s (layer %lld, expert %lld) is not a gate_proj, up_proj "
                         "or down_proj weight", nm->s.c_str(), (long long)l, (long long)x);
        } else {
            role = count[ex];           // the engine's rule: entry order gate, up, down
            DS4F_REQUIRE(role < 3, "pool layout: layer %lld expert %lld has more than three tensors", (long long)l,
                         (long long)x);
        }
        count[ex]++;
        DS4F_REQUIRE(!(seen[ex] & (1u << role)), "pool layout: layer %lld expert %lld gives %s twice", (long long)l,
                     (long long)x, kRoleName[role]);
        seen[ex] |= (uint8_t)(1u << role);
        const int64_t R = role == 2 ? H : M, C = role == 2 ? M : H;
        DS4F_REQUIRE(shp->a.size() == 2 && shp->a[0].is_int && shp->a[1].is_int && shp->a[0].i == R &&
                         shp->a[1].i == C,
                     "pool layout: layer %lld expert %lld %s: shape is not [%lld, %lld]", (long long)l, (long long)x,
                     kRoleName[role], (long long)R, (long long)C);
        DS4F_REQUIRE(vn == vb && sn == sb,
                     "pool layout: layer %lld expert %lld %s: %lld value + %lld scale bytes, the model's format "
                     "has %lld + %lld",
                     (long long)l, (long long)x, kRoleName[role], (long long)vn, (long long)sn, (long long)vb,
                     (long long)sb);
        DS4F_REQUIRE(vo >= 0 && so >= 0, "pool layout: tensor L%lld E%lld at a negative offset", (long long)l,
                     (long long)x);
        const int64_t slot_off = 24 + (int64_t)ex * nb;
        const int64_t rv = vo - slot_off, rs = so - slot_off;
        DS4F_REQUIRE(rv >= 0 && rs >= 0 && rv + vn <= nb && rs + sn <= nb,
                     "pool layout: tensor L%lld E%lld out of slot bounds (rel_v=%lld rel_s=%lld, slot=%lld)",
                     (long long)l, (long long)x, (long long)rv, (long long)rs, (long long)nb);
        off[ex * 6 + 2 * role] = vo;
        off[ex * 6 + 2 * role + 1] = so;
    }
    for (size_t ex = 0; ex < seen.size(); ex++)
        for (int r = 0; r < 3; r++)
            DS4F_REQUIRE(seen[ex] & (1u << r), "pool layout: layer %d expert %d lacks %s", (int)(ex / E),
                         (int)(ex % E), kRoleName[r]);
    *nbytes = nb;
    return 0;
}

}  // namespace ds4f

extern "C" {

int ds4f_pool_layout_plan(const char *json_path, int fmt, int hidden, int moe_inter, int n_layers, int n_experts,
                          int64_t *offsets, int64_t *expert_nbytes) {
    DS4F_REQUIRE(json_path && n_layers > 0 && n_experts > 0, "pool_layout_plan: bad arguments");
    std::vector<int64_t> off;
    int64_t nb = 0;
    if (ds4f::pool_plan(json_path, fmt, hidden, moe_inter, n_layers, n_experts, off, &nb)) return -1;
    if (offsets) memcpy(offsets, off.data(), off.size() * sizeof(int64_t));
    if (expert_nbytes) *expert_nbytes = nb;
    return 0;
}

int ds4f_gpu_pool_load_json(Ds4fGpuModel *h, const char *pool_path, const char *json_path) {
    using namespace ds4f;
    DS4F_REQUIRE(h && pool_path && json_path, "pool_load_json: null argument");
    Model &m = h->m;
    DS4F_REQUIRE(!m.cache, "pool_load_json: a streaming model reads its experts from the caller's host pool");
    const int L = m.d.n_layers, E = m.d.n_experts;
    std::vector<int64_t> off;
    int64_t nb = 0;
    if (pool_plan(json_path, m.d.fmt, m.d.hidden, m.d.moe_inter, L, E, off, &nb)) return -1;
    int fd = open(pool_path, O_RDONLY);
    DS4F_REQUIRE(fd >= 0, "pool_load_json: cannot open %s", pool_path);
    uint8_t hdr[24];
    if (pread(fd, hdr, 24, 0) != 24) { close(fd); set_error("pool_load_json: short header in %s", pool_path); return -1; }
    auto rdu = [&](int o) { uint64_t v = 0; for (int i = 7; i >= 0; i--) v = (v << 8) | hdr[o + i]; return v; };
    const off_t sz = lseek(fd, 0, SEEK_END);
    if ((int64_t)rdu(0) != nb || (int64_t)rdu(8) != L || (int64_t)rdu(16) != E ||
        sz != (off_t)(24 + nb * (int64_t)L * E)) {
        close(fd);
        set_error("pool_load_json: %s header (%llu B, %llu x %llu) or size %lld disagrees with its layout "
                  "(%lld B, %d x %d)", pool_path, (unsigned long long)rdu(0), (unsigned long long)rdu(8),
                  (unsigned long long)rdu(16), (long long)sz, (long long)nb, L, E);
        return -1;
    }
    // k whole source slots per read, permuted on the host into k slots of
    // this library's layout, copied up while the next read runs
    const int64_t dnb = m.slot.nbytes;
    const int k = (int)std::max<int64_t>(1, std::min<int64_t>(m.d.expert_count, ((int64_t)32 << 20) / std::max(nb, dnb)));
    uint8_t *src = nullptr, *dst[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int rc = -1;
    if (cudaMallocHost((void **)&src, (size_t)k * nb) != cudaSuccess ||
        cudaMallocHost((void **)&dst[0], (size_t)k * dnb) != cudaSuccess ||
        cudaMallocHost((void **)&dst[1], (size_t)k * dnb) != cudaSuccess ||
        cudaEventCreate(&ev[0]) != cudaSuccess || cudaEventCreate(&ev[1]) != cudaSuccess) {
        set_error("pool_load_json: pinned staging allocation failed");
        goto out;
    }
    {
        int b = 0;
        for (int l = 0; l < L; l++)
            for (int x0 = 0; x0 < m.d.expert_count; x0 += k) {
                const int n = std::min(k, m.d.expert_count - x0);
                const int64_t first = (int64_t)l * E + m.d.expert_first + x0;
                const int64_t base = 24 + first * nb;
                size_t got = 0;
                while (got < (size_t)(n * nb)) {
                    ssize_t r = pread(fd, src + got, (size_t)n * nb - got, base + got);
                    if (r <= 0) { set_error("pool_load_json: read error in %s", pool_path); goto out; }
                    got += (size_t)r;
                }
                if (cudaEventSynchronize(ev[b]) != cudaSuccess) { set_error("pool_load_json: event"); goto out; }
                for (int j = 0; j < n; j++) {
                    const int64_t *o = &off[(size_t)(first + j) * 6];
                    const uint8_t *s = src + (int64_t)j * nb;
                    const int64_t slot_file = base + (int64_t)j * nb;    // in-slot offsets were checked
                    uint8_t *d = dst[b] + (int64_t)j * dnb;
                    for (int r = 0; r < 3; r++) {
                        memcpy(d + m.slot.rel_v[r], s + (o[2 * r] - slot_file),
                               (size_t)(m.slot.rel_s[r] - m.slot.rel_v[r]));
                        const int64_t send = r < 2 ? m.slot.rel_v[r + 1] : dnb;
                        memcpy(d + m.slot.rel_s[r], s + (o[2 * r + 1] - slot_file), (size_t)(send - m.slot.rel_s[r]));
                    }
                }
                uint8_t *dev = m.pool + ((int64_t)l * m.d.expert_count + x0) * dnb;
                if (cudaMemcpyAsync(dev, dst[b], (size_t)n * dnb, cudaMemcpyHostToDevice, m.stream) != cudaSuccess ||
                    cudaEventRecord(ev[b], m.stream) != cudaSuccess) {
                    set_error("pool_load_json: copy failed");
                    goto out;
                }
                b ^= 1;
            }
        if (m.d.fmt == DS4F_FMT_FP8)
            for (int64_t i = 0; i < (int64_t)L * m.d.expert_count; i++)
                for (int t = 0; t < 3; t++)
                    if (launch_f8_canon(m.pool + i * dnb + m.slot.rel_v[t], m.slot.rel_s[t] - m.slot.rel_v[t],
                                        m.stream))
                        goto out;
        if (cudaStreamSynchronize(m.stream) != cudaSuccess) { set_error("pool_load_json: sync failed"); goto out; }
        rc = 0;
    }
out:
    cudaStreamSynchronize(m.stream);
    if (ev[0]) cudaEventDestroy(ev[0]);
    if (ev[1]) cudaEventDestroy(ev[1]);
    if (src) cudaFreeHost(src);
    if (dst[0]) cudaFreeHost(dst[0]);
    if (dst[1]) cudaFreeHost(dst[1]);
    close(fd);
    return rc;
}

}  // extern "C"
