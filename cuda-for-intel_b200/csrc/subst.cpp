// subst.cpp -- substitution policy, kernel table and launch router of libcfi_b200.so.
//
// Host-side restatement (C++) of cuda-for-intel src/subst/mod.rs and src/cuda/subst_hook.rs for
// the real CUDA driver: a recognised ggml kernel launch runs the precompiled sm_100a replacement;
// any build, probe or launch failure marks the plan failed and the caller's stock CUfunction
// runs instead (through cuLaunchKernel, looked up with cudaGetDriverEntryPoint so the library
// loads on machines without a GPU driver).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <cctype>
#include <tuple>

#include "cfi_kernels.h"
#include "subst_host.hpp"

namespace cfi {

// ---------------------------------------------------------------------------------------------
// logging (subst_hook.rs logs every decision; here only when CFI_SUBST_LOG is set)
// ---------------------------------------------------------------------------------------------
static void logf_(const char* fmt, ...) {
    static int on = -1;
    if (on < 0) {
        const char* v = getenv("CFI_SUBST_LOG");
        on = v && *v && strcmp(v, "0") != 0;
    }
    if (!on) return;
    va_list ap;
    va_start(ap, fmt);
    fputs("cfi-subst: ", stderr);
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
}

static const char* env2(const char* a, const char* b) {
    const char* v = getenv(a);
    return v ? v : getenv(b);
}

static std::string lower_trim(const std::string& s) {
    size_t i = 0, j = s.size();
    while (i < j && isspace((unsigned char)s[i])) i++;
    while (j > i && isspace((unsigned char)s[j - 1])) j--;
    std::string r = s.substr(i, j - i);
    for (auto& c : r) c = (char)tolower((unsigned char)c);
    return r;
}

// ---------------------------------------------------------------------------------------------
// Switch (mod.rs:57-113)
// ---------------------------------------------------------------------------------------------
Switch Switch::parse(const std::string& text) {
    Switch s;
    size_t pos = 0;
    while (pos <= text.size()) {
        size_t comma = text.find(',', pos);
        if (comma == std::string::npos) comma = text.size();
        std::string item = lower_trim(text.substr(pos, comma - pos));
        pos = comma + 1;
        if (item.empty()) continue;
        if (item == "none" || item == "0" || item == "off") {
            s.all = s.aut = false;
            s.items.clear();
            s.denied.clear();
        } else if (item == "all" || item == "1" || item == "on") {
            s.all = true;
        } else if (item == "auto") {
            s.aut = true;
        } else if (item[0] == '-' && item.size() > 1) {
            s.denied.push_back(item.substr(1));
        } else {
            s.items.push_back(item);
        }
    }
    return s;
}

Switch Switch::from_env() {
    const char* v = env2("CFI_SUBST", "CUDA_FOR_INTEL_SUBST");
    return parse(v ? v : "auto");
}

static bool item_matches(const std::string& i, const std::string& family, const char* ty) {
    if (i == family) return true;
    if (!ty) return false;
    return i.size() > family.size() + 1 && i.compare(0, family.size(), family) == 0 && i[family.size()] == ':' &&
           i.substr(family.size() + 1) == ty;
}

bool Switch::allows(const std::string& family, const char* ty) const {
    if (all) return true;
    for (auto& i : items)
        if (item_matches(i, family, ty)) return true;
    return false;
}

bool Switch::denies(const std::string& family, const char* ty) const {
    for (auto& d : denied)
        if (item_matches(d, family, ty)) return true;
    return false;
}

// ---------------------------------------------------------------------------------------------
// demangle (mod.rs:129-171).  Besides the literal template arguments the reference parses
// (L<type><value>E), builtin and named *type* arguments are accepted (rope_neox<..., float>,
// soft_max_f32<..., __half>); expressions (X...E) and packs still give no match.
// ---------------------------------------------------------------------------------------------
static bool source_name(const std::string& s, size_t& pos, std::string& out) {
    size_t d = pos;
    while (d < s.size() && isdigit((unsigned char)s[d])) d++;
    if (d == pos) return false;
    size_t n = strtoull(s.substr(pos, d - pos).c_str(), nullptr, 10);
    if (n == 0 || s.size() - d < n) return false;
    out = s.substr(d, n);
    pos = d + n;
    return true;
}

std::optional<Mangled> demangle(const std::string& name) {
    if (name.compare(0, 2, "_Z") != 0) return std::nullopt;
    size_t pos = 2;
    Mangled m;
    if (!source_name(name, pos, m.base)) return std::nullopt;
    if (pos < name.size() && name[pos] == 'I') {
        pos++;
        for (;;) {
            if (pos >= name.size()) return std::nullopt;
            char c = name[pos];
            if (c == 'E') break;
            if (c == 'L') {
                pos++;
                TArg a{TArg::Int, 0, ""};
                if (pos < name.size() && isdigit((unsigned char)name[pos])) {
                    if (!source_name(name, pos, a.name)) return std::nullopt;
                    a.kind = TArg::Enum;
                } else {
                    if (pos >= name.size()) return std::nullopt;
                    pos++;  // builtin type code of the literal
                }
                bool neg = pos < name.size() && name[pos] == 'n';
                if (neg) pos++;
                size_t d = pos;
                while (d < name.size() && isdigit((unsigned char)name[d])) d++;
                if (d == pos) return std::nullopt;
                a.value = strtoll(name.substr(pos, d - pos).c_str(), nullptr, 10);
                if (neg) a.value = -a.value;
                pos = d;
                if (pos >= name.size() || name[pos] != 'E') return std::nullopt;
                pos++;
                m.targs.push_back(a);
            } else if (isdigit((unsigned char)c)) {
                TArg a{TArg::Type, 0, ""};
                if (!source_name(name, pos, a.name)) return std::nullopt;
                m.targs.push_back(a);
            } else if (strchr("fdijlmxybcahstv", c)) {
                m.targs.push_back(TArg{TArg::Type, 0, std::string(1, c)});
                pos++;
            } else {
                return std::nullopt;
            }
        }
    }
    return m;
}

// ---------------------------------------------------------------------------------------------
// layouts (mod.rs:189-291)
// ---------------------------------------------------------------------------------------------
static cfi_param P(int kind, uint16_t a = 0, uint16_t b = 0, uint8_t c = 0) {
    cfi_param p;
    p.kind = kind;
    p.a = a;
    p.b = b;
    p.c = c;
    return p;
}
static cfi_param ptr() { return P(CFI_P_PTR); }
static cfi_param u32() { return P(CFI_P_U32); }
static cfi_param u64() { return P(CFI_P_U64); }
static cfi_param f32() { return P(CFI_P_F32); }
static cfi_param u3() { return P(CFI_P_WORDS, 3, 4, 0); }

size_t param_bytes(const cfi_param& p) {
    switch (p.kind) {
    case CFI_P_U8: return 1;
    case CFI_P_U16: return 2;
    case CFI_P_U32:
    case CFI_P_F32: return 4;
    case CFI_P_U64:
    case CFI_P_PTR: return 8;
    case CFI_P_WORDS: return (size_t)p.a * 4;
    case CFI_P_STAGED: return 8;  // the kernel receives a pointer to the staged copy
    default: return 0;
    }
}

std::string layout_debug(const cfi_param* p, int n) {
    std::string s = "[";
    char buf[96];
    for (int i = 0; i < n; i++) {
        if (i) s += ", ";
        switch (p[i].kind) {
        case CFI_P_U8: s += "U8"; break;
        case CFI_P_U16: s += "U16"; break;
        case CFI_P_U32: s += "U32"; break;
        case CFI_P_F32: s += "F32"; break;
        case CFI_P_U64: s += "U64"; break;
        case CFI_P_PTR: s += "GlobalPtr"; break;
        case CFI_P_WORDS:
            snprintf(buf, sizeof buf, "Words { words: %u, align: %u, trim: %u }", p[i].a, p[i].b, p[i].c);
            s += buf;
            break;
        case CFI_P_STAGED:
            snprintf(buf, sizeof buf, "Staged { bytes: %u, align: %u }", p[i].a, p[i].b);
            s += buf;
            break;
        default: s += "?"; break;
        }
    }
    return s + "]";
}

uint64_t layout_hash(const cfi_param* p, int n) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (unsigned char b : layout_debug(p, n)) {
        h ^= b;
        h *= 0x100000001b3ull;
    }
    return h;
}

static bool param_eq(const cfi_param& a, const cfi_param& b) {
    if (a.kind != b.kind) return false;
    if (a.kind == CFI_P_WORDS) return a.a == b.a && a.b == b.b && a.c == b.c;
    if (a.kind == CFI_P_STAGED) return a.a == b.a && a.b == b.b;
    return true;
}

Layout layout_for(int kernel, uint32_t aux) {
    Layout v;
    switch (kernel) {
    case CFI_K_MMVQ:  // mod.rs:214-218
        v = {ptr(), ptr(), ptr(), ptr(), u32(), u3(), u32(), u32(), u32(), u3(), u32(), u32(), u32(), u3(), u32(), u32(), u32()};
        break;
    case CFI_K_QUANTIZE_Q8_1:  // mod.rs:220-223
        v = {ptr(), ptr(), u64(), u64(), u64(), u64(), u64(), u32(), u3()};
        break;
    case CFI_K_MMQ:  // mod.rs:225-230
        v.assign(6, ptr());
        v.insert(v.end(), 17, u32());
        break;
    case CFI_K_MMQ_FIXUP:  // mod.rs:232-237
        v.assign(4, ptr());
        v.insert(v.end(), 9, u32());
        break;
    case CFI_K_QUANTIZE_MMQ:  // (x, ids, vy, i64 ne00, s01, s02, s03, ne0, int ne1, int ne2)
        v = {ptr(), ptr(), ptr(), u64(), u64(), u64(), u64(), u64(), u32(), u32()};
        break;
    case CFI_K_RMS_NORM:  // PKfPfixxxfS1_xxx5uint3S3_S3_S3_S1_xxxS3_S3_S3_S3_
        v = {ptr(), ptr(), u32(), u64(), u64(), u64(), f32(), ptr(), u64(), u64(), u64(), u3(), u3(), u3(), u3(),
             ptr(), u64(), u64(), u64(), u3(), u3(), u3(), u3()};
        break;
    case CFI_K_RMS_NORM_PLAIN:  // PKfPfiiilllf
        v = {ptr(), ptr(), u32(), u32(), u32(), u64(), u64(), u64(), f32()};
        break;
    case CFI_K_ROPE_NEOX:  // PKT1_PS0_iiiiiPKifff14rope_corr_dimsfPKf
        v = {ptr(), ptr(), u32(), u32(), u32(), u32(), u32(), ptr(), f32(), f32(), f32(), P(CFI_P_WORDS, 2, 4, 0), f32(), ptr()};
        break;
    case CFI_K_SOFT_MAX:  // PKfPKT2_S1_Pf15soft_max_params (128-byte struct, 8-aligned)
        v = {ptr(), ptr(), ptr(), ptr(), P(CFI_P_WORDS, 32, 8, 0)};
        break;
    case CFI_K_FATTN:  // mod.rs:239-242: 8 pointers, 29 scalars (nb13, nb23, nb33 int64)
        v.assign(8, ptr());
        v.insert(v.end(), {f32(), f32(), f32(), f32(), u32(), f32()});
        v.insert(v.end(), 13, u32());
        v.insert(v.end(), {u64(), u32(), u32(), u64(), u32(), u32(), u32(), u32(), u32(), u64()});
        break;
    case CFI_K_FATTN_FIXUP:  // mod.rs:244-247: dst, dst_fixup, ne01, ne02, ne03, ne11
        v = {ptr(), ptr(), u32(), u32(), u32(), u32()};
        break;
    }
    (void)aux;
    return v;
}

int nparams_for(int kernel, uint32_t aux) { return (int)layout_for(kernel, aux).size(); }

// mod.rs:259-291, plus a size-only rule: a B200 driver hook learns parameter sizes
// (cuFuncGetParamInfo), not PTX types, so a layout whose every parameter has the expected size
// also matches.
static bool layout_matches(int kernel, uint32_t ncols, const cfi_param* params, int n, const Layout& expected) {
    if ((size_t)n != expected.size()) return false;
    bool exact = true;
    for (int i = 0; i < n; i++) exact = exact && param_eq(params[i], expected[i]);
    if (exact) return true;
    if (kernel == CFI_K_MMQ || kernel == CFI_K_MMQ_FIXUP || kernel == CFI_K_FATTN || kernel == CFI_K_FATTN_FIXUP) {
        int lead = kernel == CFI_K_MMQ ? 6 : kernel == CFI_K_MMQ_FIXUP ? 4 : kernel == CFI_K_FATTN ? 8 : 2;
        bool ok = true;
        for (int i = 0; i < n && ok; i++)
            ok = param_eq(params[i], expected[i]) || (i < lead && (params[i].kind == CFI_P_U64 || params[i].kind == CFI_P_PTR));
        if (ok) return true;
    }
    if (kernel == CFI_K_MMVQ && ncols > 1 && params[2].kind == CFI_P_U64) {
        bool ok = true;
        for (int i = 0; i < n && ok; i++) ok = i == 2 || param_eq(params[i], expected[i]);
        if (ok) return true;
    }
    for (int i = 0; i < n; i++)
        if (param_bytes(params[i]) != param_bytes(expected[i]) || param_bytes(params[i]) == 0) return false;
    return true;
}

const char* type_name(uint32_t ty) {
    switch (ty) {
    case 2: return "q4_0";
    case 6: return "q5_0";
    case 8: return "q8_0";
    case 12: return "q4_k";
    case 13: return "q5_k";
    case 14: return "q6_k";
    default: return nullptr;
    }
}

static bool mmvq_supported(uint32_t ty) { return ty == 2 || ty == 8 || ty == 12 || ty == 14; }
static bool mmq_supported(uint32_t ty) { return ty == 2 || ty == 6 || ty == 8 || ty == 12 || ty == 13 || ty == 14; }

// mod.rs:196-212: every known kernel is in `auto` (the B200 row kernels too).
static bool auto_ok(int kernel, uint32_t ty) {
    if (kernel == CFI_K_MMQ || kernel == CFI_K_MMQ_FIXUP) return mmq_supported(ty);
    return true;
}

// ---------------------------------------------------------------------------------------------
// decode-fast knob (mod.rs:323-387)
// ---------------------------------------------------------------------------------------------
bool mmvq_fast_is_opt_out(const std::string& t) {
    std::string s = lower_trim(t);
    return s == "0" || s == "off" || s == "false" || s == "no" || s == "none";
}

cfi_fast mmvq_fast_default(uint32_t ty) {
    cfi_fast f;
    f.rows = 4;
    f.warps = 1;
    f.unroll = 2;
    f.wide = (ty == 8 || ty == 12 || ty == 14) ? 1 : 0;
    return f;
}

static bool pow2(uint32_t v) { return v && !(v & (v - 1)); }

std::optional<cfi_fast> mmvq_fast_from(const char* text_c, uint32_t ty) {
    std::string text = lower_trim(text_c ? text_c : "");
    if (mmvq_fast_is_opt_out(text)) return std::nullopt;
    if (text.empty() || text == "1" || text == "on" || text == "true" || text == "yes" || text == "auto")
        return mmvq_fast_default(ty);
    bool wide = false;
    std::string body = text;
    if (!body.empty() && body.back() == 'w') {
        wide = true;
        body.pop_back();
    }
    std::vector<std::string> parts;
    size_t pos = 0;
    for (;;) {
        size_t e = body.find_first_of(",x", pos);
        parts.push_back(body.substr(pos, e == std::string::npos ? std::string::npos : e - pos));
        if (e == std::string::npos) break;
        pos = e + 1;
    }
    if (parts.size() != 3) return std::nullopt;
    uint32_t v[3];
    for (int i = 0; i < 3; i++) {
        std::string p = lower_trim(parts[i]);
        if (p.empty() || p.find_first_not_of("0123456789") != std::string::npos || p.size() > 9) return std::nullopt;
        v[i] = (uint32_t)strtoul(p.c_str(), nullptr, 10);
    }
    cfi_fast f;
    f.rows = v[0];
    f.warps = v[1];
    f.unroll = v[2];
    f.wide = wide && (ty == 8 || ty == 12 || ty == 14);
    if (pow2(f.rows) && pow2(f.warps) && f.rows * f.warps <= 32 && f.warps <= 8 && f.unroll >= 1 && f.unroll <= 8) return f;
    return std::nullopt;
}

static std::optional<cfi_fast> mmvq_fast_env(uint32_t ty) {
    const char* text = env2("CFI_MMVQ_FAST", "CUDA_FOR_INTEL_MMVQ_FAST");
    auto f = mmvq_fast_from(text, ty);
    static bool warned = false;
    if (!f && text && !mmvq_fast_is_opt_out(text) && !warned) {
        warned = true;
        logf_("CFI_MMVQ_FAST=%s not understood; using the stock-order mmvq", text);
    }
    return f;
}

std::string mmvq_key(uint32_t ty, uint32_t ncols, const cfi_fast* f, uint32_t nwarps) {
    char buf[64];
    if (f)
        snprintf(buf, sizeof buf, "mmvq:t%u:c%u:fast%ux%ux%u%s", ty, ncols, f->rows, f->warps, f->unroll, f->wide ? "w" : "");
    else
        snprintf(buf, sizeof buf, "mmvq:t%u:c%u:w%u", ty, ncols, nwarps);
    return buf;
}

uint32_t ggml_mmvq_nwarps(uint32_t ncols) { return ncols <= 4 ? 4 : 2; }  // refs.rs:290-292

// ---------------------------------------------------------------------------------------------
// decide (mod.rs:397-466)
// ---------------------------------------------------------------------------------------------
int decide(const std::string& name, const cfi_param* params, int nparams, const Switch& sw, cfi_plan* out,
           std::string* why) {
    if (sw.is_none()) return CFI_NOT_APPLICABLE;
    auto m = demangle(name);
    if (!m) return CFI_NOT_APPLICABLE;
    const auto& t = m->targs;
    int kernel = 0;
    uint32_t ty = 0, ncols = 0, aux = 0;
    std::string family;
    const char* tname = nullptr;
    auto is_enum = [&](size_t i, const char* e) { return i < t.size() && t[i].kind == TArg::Enum && t[i].name == e; };
    auto is_int = [&](size_t i) { return i < t.size() && t[i].kind == TArg::Int; };
    auto is_type = [&](size_t i) { return i < t.size() && t[i].kind == TArg::Type; };
    const std::string& b = m->base;
    if (b == "mul_mat_vec_q" && t.size() == 2 && is_enum(0, "ggml_type") && is_int(1)) {
        ty = (uint32_t)t[0].value;
        int64_t nc = t[1].value;
        if (!type_name(ty) || !mmvq_supported(ty) || nc < 1 || nc > 8) return CFI_NOT_APPLICABLE;
        kernel = CFI_K_MMVQ;
        ncols = (uint32_t)nc;
        family = "mmvq";
        tname = type_name(ty);
    } else if (b == "mul_mat_q" && t.size() == 3 && is_enum(0, "ggml_type") && is_int(1) && is_int(2) &&
               mmq_supported((uint32_t)t[0].value)) {
        kernel = CFI_K_MMQ;
        ty = (uint32_t)t[0].value;
        aux = (uint32_t)t[1].value;
        family = "mmq";
        tname = type_name(ty);
    } else if (b == "mul_mat_q_stream_k_fixup" && t.size() == 3 && is_enum(0, "ggml_type") && is_int(1) && is_int(2) &&
               mmq_supported((uint32_t)t[0].value)) {
        kernel = CFI_K_MMQ_FIXUP;
        ty = (uint32_t)t[0].value;
        aux = (uint32_t)t[1].value;
        family = "mmq";
        tname = type_name(ty);
    } else if (b == "quantize_q8_1" && t.empty()) {
        kernel = CFI_K_QUANTIZE_Q8_1;
        family = "quantize_q8_1";
    } else if (b == "quantize_mmq_q8_1" && t.size() == 1 && is_enum(0, "mmq_q8_1_ds_layout") &&
               (t[0].value == 0 || t[0].value == 1)) {
        kernel = CFI_K_QUANTIZE_MMQ;
        ty = (uint32_t)t[0].value;  // 0 = D4, 1 = DS4
        family = "quantize_mmq";
    } else if (b == "rms_norm_f32" && t.size() == 3 && is_int(0) && is_int(1) && is_int(2)) {
        kernel = CFI_K_RMS_NORM;
        aux = (uint32_t)((t[1].value ? 1 : 0) | (t[2].value ? 2 : 0));
        family = "rms_norm";
    } else if (b == "rms_norm_f32" && t.size() == 1 && is_int(0)) {
        kernel = CFI_K_RMS_NORM_PLAIN;
        family = "rms_norm";
    } else if (b == "rope_neox" && t.size() == 3 && is_int(0) && is_int(1) && is_type(2) && t[2].name == "f") {
        kernel = CFI_K_ROPE_NEOX;
        aux = (uint32_t)((t[0].value ? 1 : 0) | (t[1].value ? 2 : 0));
        family = "rope";
    } else if (b == "soft_max_f32" && t.size() == 4 && is_int(0) && is_int(1) && is_int(2) && is_type(3) &&
               (t[3].name == "f" || t[3].name == "__half")) {
        kernel = CFI_K_SOFT_MAX;
        aux = t[3].name == "__half" ? 1 : 0;
        family = "soft_max";
    } else if (b == "flash_attn_ext_f16" && t.size() == 8 && is_int(0) && is_int(1) && is_int(2) && is_int(3) &&
               is_int(4) && is_int(5) && is_int(6) && is_int(7) && t[0].value == t[1].value &&
               (t[0].value == 64 || t[0].value == 128) && t[6].value == 0 && t[7].value == 0) {
        // mod.rs:420-425: equal K/Q and V head sizes 64 or 128, no logit softcap, no MLA
        kernel = CFI_K_FATTN;
        aux = (uint32_t)t[0].value;
        family = "fattn";
    } else if (b == "flash_attn_stream_k_fixup" && t.size() == 3 && is_int(0) && is_int(1) && is_int(2)) {
        kernel = CFI_K_FATTN_FIXUP;
        aux = (uint32_t)t[0].value;
        family = "fattn";
    } else {
        return CFI_NOT_APPLICABLE;
    }
    if (sw.denies(family, tname)) return CFI_NOT_APPLICABLE;
    if (!(sw.allows(family, tname) || (sw.aut && auto_ok(kernel, ty)))) return CFI_NOT_APPLICABLE;
    Layout expected = layout_for(kernel, aux);
    if (!layout_matches(kernel, ncols, params, nparams, expected)) {
        if (why) {
            char buf[512];
            snprintf(buf, sizeof buf, "%s: parameter layout %016llx differs from expected %016llx", name.c_str(),
                     (unsigned long long)layout_hash(params, nparams),
                     (unsigned long long)layout_hash(expected.data(), (int)expected.size()));
            *why = buf;
        }
        return CFI_MISMATCH;
    }
    memset(out, 0, sizeof *out);
    out->kernel = kernel;
    out->ty = ty;
    out->ncols = ncols;
    out->aux = aux;
    out->layout_hash = layout_hash(params, nparams);
    if (kernel == CFI_K_MMVQ) {
        const char* nw = env2("CFI_SUBST_NWARPS", "CUDA_FOR_INTEL_SUBST_NWARPS");
        if (nw) {
            char* end = nullptr;
            unsigned long v = strtoul(nw, &end, 10);
            if (end && *end == 0 && end != nw && pow2((uint32_t)v) && v >= 1 && v <= 32) out->nwarps = (uint32_t)v;
        }
        if (ncols == 1) {
            auto f = mmvq_fast_env(ty);
            if (f) {
                out->has_fast = 1;
                out->fast = *f;
            }
        }
    }
    std::string key;
    switch (kernel) {
    case CFI_K_MMVQ: key = mmvq_key(ty, ncols, out->has_fast ? &out->fast : nullptr, out->nwarps); break;
    case CFI_K_QUANTIZE_Q8_1: key = "quantize_q8_1"; break;
    case CFI_K_MMQ: key = "mmq:t" + std::to_string(ty); break;
    case CFI_K_MMQ_FIXUP: key = "mmq_fixup:t" + std::to_string(ty); break;
    case CFI_K_QUANTIZE_MMQ: key = "quantize_mmq:l" + std::to_string(ty); break;
    case CFI_K_RMS_NORM: key = "rms_norm:m" + std::to_string(aux & 1) + "a" + std::to_string(aux >> 1); break;
    case CFI_K_RMS_NORM_PLAIN: key = "rms_norm_plain"; break;
    case CFI_K_ROPE_NEOX: key = "rope_neox:f" + std::to_string(aux & 1) + "ff" + std::to_string(aux >> 1); break;
    case CFI_K_SOFT_MAX: key = aux ? "soft_max:f16" : "soft_max:f32"; break;
    case CFI_K_FATTN: key = "fattn:d" + std::to_string(aux); break;
    case CFI_K_FATTN_FIXUP: key = "fattn_fixup"; break;
    }
    snprintf(out->key, sizeof out->key, "%s", key.c_str());
    return CFI_SUBSTITUTE;
}

// ---------------------------------------------------------------------------------------------
// geometry (mod.rs:509-565), re-designed for the B200 kernels
// ---------------------------------------------------------------------------------------------
static int sm_count() {  // of the current device, cached per device (148 without one)
    static std::atomic<int> n[64];
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    if (dev >= 0 && dev < 64 && n[dev].load() > 0) return n[dev].load();
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
        cudaGetLastError();
        v = 148;
    }
    if (dev >= 0 && dev < 64) n[dev].store(v);
    return v;
}

static uint64_t rd_le(const void* p, size_t n) {
    uint64_t v = 0;
    memcpy(&v, p, n < 8 ? n : 8);
    return v;
}

std::vector<uint64_t> arg_values(const cfi_plan& plan, void** args) {
    Layout l = layout_for(plan.kernel, plan.aux);
    std::vector<uint64_t> v(l.size(), 0);
    if (!args) return v;
    for (size_t i = 0; i < l.size(); i++) v[i] = args[i] ? rd_le(args[i], param_bytes(l[i])) : 0;
    return v;
}

static bool block_is(const uint32_t b[3], uint32_t x, uint32_t y, uint32_t z) { return b[0] == x && b[1] == y && b[2] == z; }

// Numeric tuning knob from the environment, clamped to [lo, hi].
static uint32_t env_u32(const char* name, uint32_t dflt, uint32_t lo, uint32_t hi) {
    const char* v = getenv(name);
    if (!v || !*v) return dflt;
    char* end = nullptr;
    unsigned long x = strtoul(v, &end, 10);
    if (!end || *end) return dflt;
    return (uint32_t)std::min<unsigned long>(hi, std::max<unsigned long>(lo, x));
}

// Programmatic dependent launch for the native kernels (CFI_PDL=0 turns it off): each one lets
// its dependents launch early and waits for its predecessor before touching data it may produce.
static bool pdl_enabled() { return env_u32("CFI_PDL", 1, 0, 1) != 0; }

int mmq_tile_n(uint32_t ncols_dst);  // k_mmq_sm100.cu
int mmq_threads();
bool mmq_type_ok(uint32_t ty);

static int ensure_smem(const void* fn, size_t smem);

// CTAs of `fn` resident per SM at `threads` threads and `smem` dynamic shared memory (cached);
// 8 without a device (host-only contexts), so the layout does not depend on one.
static uint32_t resident_ctas(const void* fn, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void*, size_t>, uint32_t> memo;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = -1;
    }
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_tuple(dev, fn, smem);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    int n = 0;
    if (ensure_smem(fn, smem) != 0 || cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess) {
        cudaGetLastError();
        n = 8;
    }
    memo[key] = (uint32_t)n;
    return (uint32_t)n;
}

bool map_launch(const cfi_plan& plan, const uint32_t grid[3], const uint32_t block[3], const uint64_t* vals, int nvals,
                void** args, NativeLaunch* out) {
    NativeLaunch nl;
    nl.nparams = nparams_for(plan.kernel, plan.aux);
    switch (plan.kernel) {
    case CFI_K_MMVQ: {
        if (!block_is(block, 32, ggml_mmvq_nwarps(plan.ncols), 1) || nvals < 17) return false;
        const uint32_t ncols_x = (uint32_t)vals[4], stride_col_dst = (uint32_t)vals[8];
        const uint32_t qk = (plan.ty == 12 || plan.ty == 14) ? 256 : 32;
        if (ncols_x == 0 || ncols_x % qk) return false;
        if (plan.ty == 12 && (vals[0] & 15)) return false;  // 16-byte superblock loads
        if (plan.ty != 12 && (vals[0] & 1)) return false;   // 2-byte aligned blocks
        if ((vals[1] & 3)) return false;                       // q8_1 blocks are read as words
        const uint32_t nrows = plan.ncols == 1 ? grid[0] : std::min(2 * grid[0], stride_col_dst);
        const uint32_t planes = std::max(1u, grid[1] * grid[2]);
        // CFI_MMVQ_STREAM=0 selects the row kernel for ncols <= 2 too
        // CFI_MMVQ_STREAM_MIN_KB: weight matrices smaller than this take the row kernel
        const uint64_t wkb = (uint64_t)nrows * (uint64_t)vals[6] * (plan.ty == 12 ? 144 : plan.ty == 14 ? 210 :
                                                                     plan.ty == 2 ? 18 : 34) / 1024;
        const bool stream = cfi_mmvq_streams(plan.ncols) &&
                            (cfi_mmvq_stream_only(plan.ty) ||
                             (env_u32("CFI_MMVQ_STREAM", 1, 0, 1) != 0 && wkb >= env_u32("CFI_MMVQ_STREAM_MIN_KB", 0, 0, 1u << 30)));
        nl.fn = cfi_native_mmvq(plan.ty, plan.ncols, stream);
        uint32_t chunk = 0, nstages = 0;
        bool direct = false;
        if (stream && env_u32("CFI_MMVQ_DIRECT", 0, 0, 1)) {
            // direct fill (nstages 0; CFI_MMVQ_DIRECT=1): measured slower than the bulk copies for
            // Q4_K, and no faster for Q8_0 once the weights are fetched before the wait.
            // CFI_MMVQ_DIRECT_CTAS CTAs per SM (default 2, fewer when the kernel's registers or
            // shared memory do not allow them), chunks of at most 16 KB of rows
            const uint32_t want = env_u32("CFI_MMVQ_DIRECT_CTAS", 2, 1, 8);
            uint32_t c0 = 0;
            size_t s0 = 0;
            const uint32_t g0 = std::max(1u, std::min(nrows, (uint32_t)(sm_count() * want) / planes));
            const void* dfn = cfi_native_mmvq_direct(plan.ty, plan.ncols);
            if (dfn && cfi_mmvq_direct_layout(plan.ty, plan.ncols, ncols_x, nrows, g0, (uint32_t)vals[6], &c0, &s0)) {
                const uint32_t per_sm = std::min(want, resident_ctas(dfn, CFI_MMVQ_THREADS, s0));
                if (per_sm > 0) {
                    nl.fn = dfn;
                    nl.grid[0] = std::max(1u, std::min(nrows, (uint32_t)(sm_count() * per_sm) / planes));
                    direct = cfi_mmvq_direct_layout(plan.ty, plan.ncols, ncols_x, nrows, nl.grid[0], (uint32_t)vals[6],
                                                    &chunk, &nl.smem);
                    nstages = 0;
                }
            }
        }
        // Q4_K with 3..8 columns: the tensor-core kernel (exact int32 block dots, fp32 scales
        // reassociated: within ~1e-7 of the reference's order); CFI_MMVQ_EXACT=1 keeps the
        // kernels that reproduce the decode-fast fp32 order bit for bit
        bool mma = false;
        // (at 1-2 columns the dp4a kernel measured faster: 3.4 against 4.9 us at 8192 x 2048 x 1)
        if (stream && !direct && plan.ty == 12 && plan.ncols >= 3 && env_u32("CFI_MMVQ_EXACT", 0, 0, 1) == 0) {
            const uint32_t per_sm = env_u32("CFI_MMVQ_STREAM_CTAS", 2, 1, 8);
            const uint32_t g1 = std::max(1u, std::min(nrows, std::max(1u, (uint32_t)(sm_count() * per_sm) / planes)));
            uint32_t c1 = 0, n1 = 0;
            size_t s1 = 0;
            if (cfi_mmvq_mma_layout(ncols_x, nrows, g1, per_sm, env_u32("CFI_MMVQ_CHUNK", 32, 1, 256),
                                    1024 * env_u32("CFI_MMVQ_STAGE_KB", 48, 4, 112), env_u32("CFI_MMVQ_STAGES", 3, 1, 4),
                                    &c1, &n1, &s1)) {
                mma = true;
                nl.fn = cfi_native_mmvq_mma(plan.ty, plan.ncols);
                nl.grid[0] = g1;
                chunk = c1;
                nstages = n1;
                nl.smem = s1;
            }
        }
        if (stream && !direct && !mma) {
            // CFI_MMVQ_STREAM_CTAS CTAs per SM shared by the channel/sample planes; chunks of
            // CFI_MMVQ_CHUNK rows within CFI_MMVQ_STAGE_KB per stage, CFI_MMVQ_STAGES stages (as
            // many as fit the CTAs' shares of the SM).  Default: 3 CTAs per SM (two 32-row stages
            // each) for 32 MB of weights and more, measured 0.77 / 0.73 of HBM on the 151936 x 896
            // Q8_0 lm_head and a 65536 x 2048 Q4_K matrix against 0.61 / 0.66 with 2 (three stages);
            // 2 below, where the launch is latency-bound (8192 x 2048 Q4_K: 3.4 against 4.5 us)
            const uint32_t ctarget = env_u32("CFI_MMVQ_CHUNK", 32, 1, 256);
            auto layout = [&](uint32_t per_sm) {
                const uint32_t cap = std::max(1u, (uint32_t)(sm_count() * per_sm) / planes);
                nl.grid[0] = std::max(1u, std::min(nrows, cap));
                cfi_mmvq_stream_layout(plan.ty, plan.ncols, ncols_x, nrows, nl.grid[0], (uint32_t)vals[6], ctarget,
                                       1024 * env_u32("CFI_MMVQ_STAGE_KB", 48, 4, 112), env_u32("CFI_MMVQ_STAGES", 3, 1, 4),
                                       per_sm, &chunk, &nstages, &nl.smem);
            };
            if (getenv("CFI_MMVQ_STREAM_CTAS")) {
                layout(env_u32("CFI_MMVQ_STREAM_CTAS", 2, 1, 8));
            } else {
                // 3 per SM only where each still holds two whole chunks (65536 x 2048 Q4_K with two
                // columns: 32.2 us with one stage of 3 CTAs, 19.5 us with 2 CTAs of three stages)
                const bool big = wkb * planes >= 32u * 1024u;
                layout(big ? 3u : 2u);
                if (big) {
                    const uint32_t per_cta = (nrows + nl.grid[0] - 1) / nl.grid[0];
                    if (nstages < 2 || chunk < std::min(ctarget, per_cta)) layout(2u);
                }
            }
        } else if (!stream) {
            const uint32_t per_sm = env_u32("CFI_MMVQ_CTAS", 4, 1, 8);
            const uint32_t cap = std::max(1u, (uint32_t)(sm_count() * per_sm) / planes);
            const uint32_t rows_per_pass = CFI_MMVQ_WARPS * cfi_mmvq_rows_per_warp(plan.ty, plan.ncols);
            const uint32_t tiles = (nrows + rows_per_pass - 1) / rows_per_pass;
            nl.grid[0] = std::max(1u, std::min(tiles, cap));
            nl.smem = cfi_mmvq_smem_bytes(plan.ty, plan.ncols, ncols_x);
        }
        if (nl.smem > (size_t)cfi_mmvq_max_smem_bytes()) return false;
        nl.block[0] = CFI_MMVQ_THREADS;
        nl.extra.push_back(nrows);
        nl.extra.push_back(chunk);
        // CFI_MMVQ_WARP_PIPE=0: the streaming kernels' CTA-wide chunk loop (bit 10 of the stage word)
        nl.extra.push_back(nstages | (nstages && env_u32("CFI_MMVQ_WARP_PIPE", 1, 0, 1) == 0 ? 0x400u : 0u));
        nl.pdl = pdl_enabled();
        nl.grid[1] = grid[1];
        nl.grid[2] = grid[2];
        break;
    }
    case CFI_K_QUANTIZE_Q8_1:
        if (!block_is(block, 256, 1, 1)) return false;
        if (nvals >= 7 && (vals[6] % 32)) return false;
        nl.fn = cfi_native_quantize_q8_1();
        nl.pdl = pdl_enabled();
        nl.grid[0] = (grid[0] + 3) / 4;
        nl.grid[1] = grid[1];
        nl.grid[2] = grid[2];
        nl.block[0] = 256;
        break;
    case CFI_K_QUANTIZE_MMQ:
        if (!block_is(block, 128, 1, 1)) return false;
        if (nvals >= 8 && (vals[7] % 128)) return false;
        nl.fn = cfi_native_quantize_mmq(plan.ty == 1);
        memcpy(nl.grid, grid, sizeof nl.grid);
        nl.block[0] = 128;
        nl.pdl = pdl_enabled();
        break;
    case CFI_K_MMQ: {
        // mod.rs:542-557: stock 32x8 threads; MoE (ids_dst / expert_bounds) keeps the stock kernel
        if (!block_is(block, 32, 8, 1) || nvals != 23 || vals[2] != 0 || vals[3] != 0) return false;
        const uint64_t nrows = vals[7], ncols_dst = vals[8], nch = vals[13], nsamples = vals[18];
        if (nrows == 0 || ncols_dst == 0 || nch == 0 || nsamples == 0 || vals[6] % 128 != 0) return false;
        if (!mmq_type_ok(plan.ty)) return false;
        const int tn = mmq_tile_n((uint32_t)ncols_dst);
        nl.grid[0] = (uint32_t)((nrows + 127) / 128);
        nl.grid[1] = (uint32_t)((ncols_dst + tn - 1) / tn);
        nl.grid[2] = (uint32_t)(nch * nsamples);
        nl.block[0] = (uint32_t)mmq_threads();
        nl.own_launch = true;
        nl.fn = reinterpret_cast<const void*>(&mmq_launch);
        break;
    }
    case CFI_K_RMS_NORM:
    case CFI_K_RMS_NORM_PLAIN:
        if (block[1] != 1 || block[2] != 1 || !pow2(block[0]) || block[0] < 32 || block[0] > 1024) return false;
        nl.fn = plan.kernel == CFI_K_RMS_NORM ? cfi_native_rms_norm(plan.aux & 1, (plan.aux >> 1) & 1) : cfi_native_rms_norm_plain();
        memcpy(nl.grid, grid, sizeof nl.grid);
        // batched launches (>= 1024 rows): one warp per row, 8 rows per CTA, the row count appended;
        // fewer rows (a decode step): one CTA per row, the order the fused decode step reproduces
        if (plan.kernel == CFI_K_RMS_NORM && (uint64_t)grid[0] * grid[1] * grid[2] >= 1024) {
            const uint32_t wpb = CFI_ROWOP_THREADS / 32;
            nl.grid[0] = (grid[0] + wpb - 1) / wpb;
            nl.extra.push_back(grid[0]);
        } else if (plan.kernel == CFI_K_RMS_NORM) {
            nl.fn = cfi_native_rms_norm_block(plan.aux & 1, (plan.aux >> 1) & 1);
        }
        nl.block[0] = CFI_ROWOP_THREADS;
        nl.pdl = pdl_enabled();
        break;
    case CFI_K_ROPE_NEOX: {
        if (!block_is(block, 1, 256, 1) || nvals < 7 || grid[2] != 1) return false;
        const uint64_t ne0 = (uint32_t)vals[2], n_dims = (uint32_t)vals[6];
        if (ne0 == 0 || (ne0 & 1) || (n_dims & 1) || n_dims > ne0) return false;
        if (ne0 > (uint64_t)cfi_rope_max_ne0()) return false;
        const uint64_t nr = grid[0];
        const uint32_t rpw = (uint32_t)cfi_rope_rows_per_warp((uint32_t)nr);
        nl.block[0] = CFI_ROWOP_THREADS;
        nl.extra.push_back((uint32_t)nr);
        if (rpw > 1) {  // large launches: a warp per rpw rows, the frequencies kept per lane
            const uint64_t rpc = (uint64_t)rpw * (CFI_ROWOP_THREADS / 32);
            nl.fn = cfi_native_rope_neox(plan.aux & 1, (plan.aux >> 1) & 1);
            nl.grid[0] = (uint32_t)((nr + rpc - 1) / rpc);
            nl.extra.push_back(rpw);
        } else {  // a thread per rotation pair
            const uint64_t pairs = nr * (ne0 / 2);
            nl.fn = cfi_native_rope_neox_pairs(plan.aux & 1, (plan.aux >> 1) & 1);
            nl.grid[0] = (uint32_t)((pairs + CFI_ROWOP_THREADS - 1) / CFI_ROWOP_THREADS);
        }
        nl.pdl = pdl_enabled();
        break;
    }
    case CFI_K_SOFT_MAX: {
        if (block[1] != 1 || block[2] != 1 || block[0] == 0 || block[0] > 1024) return false;
        int64_t ncols = 0, nb[3] = {0, 0, 0};
        if (args && args[4]) {
            memcpy(&ncols, static_cast<const uint8_t*>(args[4]) + 16, 8);
            memcpy(nb, static_cast<const uint8_t*>(args[4]) + 72, 24);  // nb11, nb12, nb13
        }
        if (args && (ncols <= 0 || ncols * 4 > 200 * 1024)) return false;
        memcpy(nl.grid, grid, sizeof nl.grid);
        nl.block[0] = CFI_ROWOP_THREADS;
        nl.pdl = pdl_enabled();
        // rows of at most 1024 columns in 16-byte pieces: one warp per row, the row in registers
        // (launches of a few rows, as a decode step's heads, keep the CTA-per-row kernel: more
        // threads per row give the shorter chain)
        bool rows = false;
        const uint64_t total_rows = (uint64_t)grid[0] * grid[1] * grid[2];
        if (args && args[0] && args[1] && args[3] && ncols % 4 == 0 && ncols <= cfi_soft_max_rows_max_cols() &&
            total_rows >= 1024) {
            uint64_t xp = 0, mp = 0, dp = 0;
            memcpy(&xp, args[0], 8);
            memcpy(&mp, args[1], 8);
            memcpy(&dp, args[3], 8);
            const uint64_t malign = (plan.aux & 1) ? 8 : 16;
            rows = ((xp | dp) & 15) == 0 && (mp % malign) == 0 &&
                   (mp == 0 || ((uint64_t)nb[0] % malign == 0 && (uint64_t)nb[1] % malign == 0 && (uint64_t)nb[2] % malign == 0));
        }
        if (rows) {
            const uint32_t wpb = CFI_ROWOP_THREADS / 32;
            nl.fn = cfi_native_soft_max_rows(plan.aux & 1);
            nl.grid[0] = (grid[0] + wpb - 1) / wpb;
            nl.extra.push_back(grid[0]);
        } else {
            nl.fn = cfi_native_soft_max(plan.aux & 1);
            nl.smem = (size_t)ncols * 4;
        }
        break;
    }
    case CFI_K_FATTN: {
        // mod.rs:27-54: stock block (32, nwarps); the native grid tiles 128 queries
        if (block[0] != 32 || block[2] != 1 || !fattn_geometry_ok(plan.aux, vals, nvals)) return false;
        const uint32_t ne01 = (uint32_t)vals[15], ne02 = (uint32_t)vals[16], ne03 = (uint32_t)vals[17];
        nl.grid[0] = (ne01 + (uint32_t)fattn_tile() - 1) / (uint32_t)fattn_tile();
        nl.grid[1] = ne02;
        nl.grid[2] = ne03;
        nl.block[0] = (uint32_t)fattn_threads();
        nl.own_launch = true;
        nl.fn = reinterpret_cast<const void*>(&fattn_launch);
        break;
    }
    default:
        return false;
    }
    if (!nl.fn) return false;
    *out = nl;
    return true;
}

const void* native_kernel(const cfi_plan& plan, std::string* why) {
    NativeLaunch nl;
    const void* fn = nullptr;
    switch (plan.kernel) {
    case CFI_K_MMVQ: fn = cfi_native_mmvq(plan.ty, plan.ncols, true); break;
    case CFI_K_QUANTIZE_Q8_1: fn = cfi_native_quantize_q8_1(); break;
    case CFI_K_QUANTIZE_MMQ: fn = cfi_native_quantize_mmq(plan.ty == 1); break;
    case CFI_K_MMQ: fn = mmq_type_ok(plan.ty) ? reinterpret_cast<const void*>(&mmq_launch) : nullptr; break;
    case CFI_K_RMS_NORM: fn = cfi_native_rms_norm(plan.aux & 1, (plan.aux >> 1) & 1); break;
    case CFI_K_RMS_NORM_PLAIN: fn = cfi_native_rms_norm_plain(); break;
    case CFI_K_ROPE_NEOX: fn = cfi_native_rope_neox(plan.aux & 1, (plan.aux >> 1) & 1); break;
    case CFI_K_SOFT_MAX: fn = cfi_native_soft_max(plan.aux & 1); break;
    case CFI_K_FATTN: fn = (plan.aux == 64 || plan.aux == 128) ? reinterpret_cast<const void*>(&fattn_launch) : nullptr; break;
    default: break;
    }
    if (!fn && why) *why = std::string("no sm_100a kernel for ") + plan.key;
    return fn;
}

// ---------------------------------------------------------------------------------------------
// context, registry and router (subst_hook.rs)
// ---------------------------------------------------------------------------------------------
enum NativeState { NS_UNKNOWN = 0, NS_READY = 1, NS_FAILED = 2 };

struct Inject {
    int nth = 0, code = 0, calls = 0;
};

// A native quantize_q8_1 held back (CFI_CTX_DEFER_Q8_1) for the mul_mat_vec_q that reads its
// output: the launch as the caller made it, with its parameters copied (16 bytes each).
struct DeferredQ81 {
    bool on = false;
    cfi_plan plan{};
    NativeLaunch nl;
    void* stock_fn = nullptr;
    uint32_t grid[3] = {}, block[3] = {}, shmem = 0;
    void* stream = nullptr;
    std::vector<uint64_t> vals;
    alignas(16) uint8_t raw[9 * 16] = {};
    void* argv[9] = {};
};

}  // namespace cfi

struct cfi_ctx {
    int device = 0;
    int flags = 0;
    std::mutex mu;
    std::map<std::string, int> natives;
    bool have_pending = false;
    uint64_t pending_dst = 0, pending_tmp = 0;
    bool fa_pending = false;  // a native FlashAttention ran: its stream-k fixup is a no-op
    uint64_t fa_dst = 0, fa_meta = 0;
    uint64_t fixup_events = 0;
    cfi::DeferredQ81 dq;
    cfi_stats stats{};
    cfi::Inject inject[5];
};

namespace cfi {

static bool injected(cfi_ctx* ctx, int site, int* code) {
    if (site <= 0 || site > 4) return false;
    Inject& in = ctx->inject[site];
    if (!in.code) return false;
    in.calls++;
    if (in.calls == in.nth) {
        *code = in.code;
        return true;
    }
    return false;
}

static bool probe_enabled() {
    const char* v = env2("CFI_SUBST_PROBE", "CUDA_FOR_INTEL_SUBST_PROBE");
    return !(v && strcmp(v, "0") == 0);
}

// Native kernel of `plan` in ctx: cached, or built (looked up) and probed once (subst_hook.rs:211-262).
static bool native_ready(cfi_ctx* ctx, const cfi_plan& plan, void* stream) {
    auto it = ctx->natives.find(plan.key);
    if (it != ctx->natives.end()) return it->second == NS_READY;
    std::string why;
    int code = 0;
    bool ok = true;
    if (injected(ctx, CFI_SITE_BUILD, &code)) {
        ok = false;
        why = "build failed (injected " + std::to_string(code) + ")";
    } else if (!native_kernel(plan, &why)) {
        ok = false;
    } else if (probe_enabled() && !(ctx->flags & CFI_CTX_FAKE)) {
        ctx->stats.probes_run++;
        if (injected(ctx, CFI_SITE_PROBE, &code)) {
            ok = false;
            why = "first-use validation: injected " + std::to_string(code);
        } else if (probe_validate(plan, stream, &why) != 0) {
            ok = false;
            why = "first-use validation: " + why;
        }
        if (!ok) ctx->stats.probes_failed++;
    }
    if (ok) {
        logf_("native %s ready", plan.key);
        ctx->natives[plan.key] = NS_READY;
    } else {
        logf_("native %s rejected, using the stock kernel: %s", plan.key, why.c_str());
        ctx->natives[plan.key] = NS_FAILED;
    }
    return ok;
}

typedef CUresult (*PFN_launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                               CUstream, void**, void**);

static PFN_launch driver_launch() {
    static PFN_launch fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuLaunchKernel", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_launch>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// The dynamic shared memory attribute is per device: remembered per (device, kernel).
static int ensure_smem(const void* fn, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, size_t> set;
    if (smem <= 48 * 1024) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = -1;
    }
    std::lock_guard<std::mutex> g(mu);
    const auto key = std::make_pair(dev, fn);
    auto it = set.find(key);
    if (it != set.end() && it->second >= smem) return 0;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    set[key] = smem;
    return 0;
}

int issue_native(const NativeLaunch& nl, const cfi_plan& plan, void** args, void* stream) {
    if (nl.own_launch) return plan.kernel == CFI_K_FATTN ? fattn_launch(plan, args, stream) : mmq_launch(plan, args, stream);
    std::vector<void*> argv(args, args + nl.nparams);
    std::vector<uint32_t> extra = nl.extra;
    for (auto& w : extra) argv.push_back(&w);
    int e = ensure_smem(nl.fn, nl.smem);
    if (e) return e;
    cudaError_t rc;
    if (nl.pdl) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(nl.grid[0], nl.grid[1], nl.grid[2]);
        cfg.blockDim = dim3(nl.block[0], nl.block[1], nl.block[2]);
        cfg.dynamicSmemBytes = nl.smem;
        cfg.stream = static_cast<cudaStream_t>(stream);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        rc = cudaLaunchKernelExC(&cfg, nl.fn, argv.data());
    } else {
        rc = cudaLaunchKernel(nl.fn, dim3(nl.grid[0], nl.grid[1], nl.grid[2]), dim3(nl.block[0], nl.block[1], nl.block[2]),
                              argv.data(), nl.smem, static_cast<cudaStream_t>(stream));
    }
    return (int)rc;
}

static int launch_stock(cfi_ctx* ctx, void* stock_fn, const uint32_t grid[3], const uint32_t block[3], uint32_t shmem,
                        void* stream, void** args) {
    int code = 0;
    if (injected(ctx, CFI_SITE_STOCK_LAUNCH, &code)) return code;
    ctx->stats.stock_launches++;
    if (ctx->flags & CFI_CTX_FAKE) return 0;
    if (!stock_fn) return (int)CUDA_ERROR_NOT_FOUND;
    PFN_launch f = driver_launch();
    if (!f) return (int)CUDA_ERROR_NOT_INITIALIZED;
    return (int)f(static_cast<CUfunction>(stock_fn), grid[0], grid[1], grid[2], block[0], block[1], block[2], shmem,
                  static_cast<CUstream>(stream), args, nullptr);
}

// ---- deferred quantize_q8_1 (CFI_CTX_DEFER_Q8_1) ----
// quantize_q8_1 values: [x, vy, ne00, s01, s02, s03, ne0, ne1, ne2]; mul_mat_vec_q values:
// [x, y, ids, dst, ncols_x, nchannels_y, stride_row_x, stride_col_y, stride_col_dst, ...].

// Launches the held-back quantize as it would have run (native, else stock).  Returns 0 or an error.
static int flush_deferred(cfi_ctx* ctx) {
    DeferredQ81& d = ctx->dq;
    if (!d.on) return 0;
    d.on = false;
    int code = 0, rc = 0;
    if (injected(ctx, CFI_SITE_NATIVE_LAUNCH, &code))
        rc = code;
    else if (!(ctx->flags & CFI_CTX_FAKE))
        rc = issue_native(d.nl, d.plan, d.argv, d.stream);
    if (rc == 0) {
        ctx->stats.native_launches++;
        return 0;
    }
    logf_("native %s launch failed (%d); using the stock kernel", d.plan.key, rc);
    if (!(ctx->flags & CFI_CTX_FAKE)) cudaGetLastError();
    ctx->natives[d.plan.key] = NS_FAILED;
    ctx->stats.native_failures++;
    return launch_stock(ctx, d.stock_fn, d.grid, d.block, d.shmem, d.stream, d.argv);
}

// Holds back a native quantize_q8_1 of up to 8 columns in one plane.  False: launch it now.
static bool defer_q81(cfi_ctx* ctx, const cfi_plan& plan, void* stock_fn, const uint32_t grid[3], const uint32_t block[3],
                      uint32_t shmem, void* stream, void** args, const std::vector<uint64_t>& v) {
    if (!(ctx->flags & CFI_CTX_DEFER_Q8_1) || v.size() != 9 || !args) return false;
    const uint64_t ne00 = v[2], ne0 = v[6], ne1 = (uint32_t)v[7];
    if (grid[2] != 1 || ne1 < 1 || ne1 > 8 || grid[1] != ne1 || ne0 == 0 || ne0 % 32 || ne00 > ne0 || (v[0] & 3) || (v[1] & 3))
        return false;
    NativeLaunch nl;
    if (!map_launch(plan, grid, block, v.data(), (int)v.size(), args, &nl) || !native_ready(ctx, plan, stream)) return false;
    DeferredQ81& d = ctx->dq;
    Layout l = layout_for(plan.kernel, plan.aux);
    if (l.size() != 9) return false;
    for (size_t i = 0; i < 9; i++) {
        const size_t n = param_bytes(l[i]);
        if (n == 0 || n > 16 || !args[i]) return false;
        memcpy(d.raw + 16 * i, args[i], n);
        d.argv[i] = d.raw + 16 * i;
    }
    d.plan = plan;
    d.nl = nl;
    d.stock_fn = stock_fn;
    memcpy(d.grid, grid, sizeof d.grid);
    memcpy(d.block, block, sizeof d.block);
    d.shmem = shmem;
    d.stream = stream;
    d.vals = v;
    d.on = true;
    return true;
}

// Runs the held-back quantize inside this GEMV launch (cfi_mmvq_stream_q81) when the GEMV reads
// exactly its output: same stream, one plane, no ids, its columns = the quantized columns, laid
// out as the quantizer writes them.  Returns 0 when launched, -1 when not applicable, else the
// launch error.
static int absorb_q81(cfi_ctx* ctx, const cfi_plan& plan, const NativeLaunch& nl, const std::vector<uint64_t>& v,
                      void** args, void* stream) {
    const DeferredQ81& d = ctx->dq;
    const uint64_t ne0 = d.vals[6];
    const bool direct = nl.fn == cfi_native_mmvq_direct(plan.ty, plan.ncols);
    if (stream != d.stream || v.size() < 17 || v[1] != d.vals[1] || v[2] != 0 || plan.ncols != (uint32_t)d.vals[7] ||
        nl.grid[1] != 1 || nl.grid[2] != 1 || (uint32_t)v[7] != ne0 / 32 || v[4] > ne0 || nl.own_launch ||
        !(direct || nl.fn == cfi_native_mmvq(plan.ty, plan.ncols, true)))
        return -1;
    // the prologue quantizes all ncols x ne0 values in every CTA: absorbed only up to
    // CFI_DEFER_MAX_VALUES of them (default 1024, one pass of the CTA's 32 eight-thread groups),
    // where that measured cheaper than a separate launch (Q8_0 4864 x 896: 3.58 against 4.92 us
    // per pair; Q4_K 8192 x 2048, two passes: slower)
    if ((uint64_t)plan.ncols * ne0 > env_u32("CFI_DEFER_MAX_VALUES", 1024, 0, 1u << 20)) return -1;
    const void* fn = cfi_native_mmvq_q81(plan.ty, plan.ncols, direct);
    if (!fn) return -1;
    int code = 0;
    if (injected(ctx, CFI_SITE_NATIVE_LAUNCH, &code)) return code;
    if (ctx->flags & CFI_CTX_FAKE) return 0;
    CfiFuseQ fq = {};
    fq.x = reinterpret_cast<const float*>(d.vals[0]);
    fq.vy = reinterpret_cast<uint8_t*>(d.vals[1]);
    fq.ne00 = (int64_t)d.vals[2];
    fq.s01 = (int64_t)d.vals[3];
    fq.nbq = (uint32_t)(ne0 / 32);
    NativeLaunch f = nl;
    f.fn = fn;
    if ((ctx->flags & CFI_CTX_CONST_WEIGHTS) && f.extra.size() == 3) f.extra[2] |= 0x100u;
    // CFI_DEFER_CLUSTER CTAs (1, 2, 4 or 8; default 1) share the quantize work of the prologue
    // through distributed shared memory (measured slower than every CTA quantizing alone)
    uint32_t cs = env_u32("CFI_DEFER_CLUSTER", 1, 1, 8);
    while (cs & (cs - 1)) cs &= cs - 1;
    f.grid[0] = (f.grid[0] + cs - 1) / cs * cs;
    std::vector<void*> argv(args, args + f.nparams);
    std::vector<uint32_t> extra = f.extra;
    for (auto& w : extra) argv.push_back(&w);
    argv.push_back(&fq);
    int e = ensure_smem(f.fn, f.smem);
    if (e) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(f.grid[0], f.grid[1], f.grid[2]);
    cfg.blockDim = dim3(f.block[0], f.block[1], f.block[2]);
    cfg.dynamicSmemBytes = f.smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (f.pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na++].val.programmaticStreamSerializationAllowed = 1;
    }
    if (cs > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cs;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return (int)cudaLaunchKernelExC(&cfg, f.fn, argv.data());
}

int launch_to(cfi_ctx* ctx, const cfi_plan* plan, void* stock_fn, const uint32_t grid[3], const uint32_t block[3],
              uint32_t shmem, void* stream, void** args) {
    std::lock_guard<std::mutex> g(ctx->mu);
    if (plan) {
        std::vector<uint64_t> vals = arg_values(*plan, args);
        if (ctx->dq.on) {
            NativeLaunch nl;
            if (plan->kernel == CFI_K_MMVQ && map_launch(*plan, grid, block, vals.data(), (int)vals.size(), args, &nl) &&
                native_ready(ctx, *plan, stream)) {
                const int rc = absorb_q81(ctx, *plan, nl, vals, args, stream);
                if (rc == 0) {
                    ctx->dq.on = false;
                    ctx->stats.native_launches += 2;
                    ctx->stats.fused_q8_1++;
                    return 0;
                }
                if (rc > 0) {
                    logf_("fused quantize_q8_1 + %s launch failed (%d); launching them separately", plan->key, rc);
                    if (!(ctx->flags & CFI_CTX_FAKE)) cudaGetLastError();
                    ctx->flags &= ~CFI_CTX_DEFER_Q8_1;
                }
            }
            const int rc = flush_deferred(ctx);
            if (rc) return rc;
        }
        if (plan->kernel == CFI_K_QUANTIZE_Q8_1 && defer_q81(ctx, *plan, stock_fn, grid, block, shmem, stream, args, vals))
            return 0;
        if (plan->kernel == CFI_K_MMQ) ctx->have_pending = false;
        if (plan->kernel == CFI_K_FATTN) ctx->fa_pending = false;
        if (plan->kernel == CFI_K_FATTN_FIXUP) {
            // [dst, dst_fixup, ...]: the native FlashAttention writes final results (fattn.rs:17-18)
            const bool skip = vals.size() == 6 && ctx->fa_pending && ctx->fa_dst == vals[0] && ctx->fa_meta == vals[1];
            if (ctx->fixup_events++ < 40) logf_("fattn fixup %s", skip ? "skipped" : "RUNS");
            if (skip) {
                ctx->fa_pending = false;
                ctx->stats.fixups_skipped++;
                return 0;
            }
        } else if (plan->kernel == CFI_K_MMQ_FIXUP) {
            // [ids, bounds, dst, tmp, ...]: only fixups of a native mul_mat_q are no-ops
            const bool skip = vals.size() == 13 && ctx->have_pending && ctx->pending_dst == vals[2] && ctx->pending_tmp == vals[3];
            if (ctx->fixup_events++ < 40) logf_("mmq fixup %s", skip ? "skipped" : "RUNS");
            if (skip) {
                ctx->have_pending = false;
                ctx->stats.fixups_skipped++;
                return 0;
            }
        } else {
            NativeLaunch nl;
            if (map_launch(*plan, grid, block, vals.data(), (int)vals.size(), args, &nl) && native_ready(ctx, *plan, stream)) {
                if ((ctx->flags & CFI_CTX_CONST_WEIGHTS) && plan->kernel == CFI_K_MMVQ && nl.extra.size() == 3 && vals[2] == 0)
                    nl.extra[2] |= 0x100u | (env_u32("CFI_MMVQ_HINT_EARLY", 0, 0, 1) ? 0x200u : 0u);  // fetch the weights before waiting on the previous kernel (and hint L2 with all of them)
                int code = 0;
                int rc = 0;
                if (injected(ctx, CFI_SITE_NATIVE_LAUNCH, &code))
                    rc = code;
                else if (!(ctx->flags & CFI_CTX_FAKE))
                    rc = issue_native(nl, *plan, args, stream);
                if (rc == 0) {
                    ctx->stats.native_launches++;
                    if (plan->kernel == CFI_K_MMQ) {
                        ctx->have_pending = true;
                        ctx->pending_dst = vals[4];
                        ctx->pending_tmp = vals[5];
                    }
                    if (plan->kernel == CFI_K_FATTN) {
                        ctx->fa_pending = true;
                        ctx->fa_dst = vals[6];
                        ctx->fa_meta = vals[7];
                    }
                    return 0;
                }
                logf_("native %s launch failed (%d); using the stock kernel", plan->key, rc);
                if (!(ctx->flags & CFI_CTX_FAKE)) cudaGetLastError();
                ctx->natives[plan->key] = NS_FAILED;
                ctx->stats.native_failures++;
            }
        }
    } else if (ctx->dq.on) {
        const int rc = flush_deferred(ctx);
        if (rc) return rc;
    }
    return launch_stock(ctx, stock_fn, grid, block, shmem, stream, args);
}

}  // namespace cfi

// =============================================================================================
// extern "C" surface
// =============================================================================================
using namespace cfi;

static void copy_out(const std::string& s, char* out, size_t len) {
    if (!out || !len) return;
    snprintf(out, len, "%s", s.c_str());
}

extern "C" {

int cfi_subst_decide(const char* mangled, const cfi_param* params, int nparams, const char* switch_text, cfi_plan* out,
                     char* why, size_t why_len) {
    if (!mangled || !out || (nparams > 0 && !params) || nparams < 0) return CFI_NOT_APPLICABLE;
    Switch sw = switch_text ? Switch::parse(switch_text) : Switch::from_env();
    std::string w;
    int r = decide(mangled, params, nparams, sw, out, &w);
    if (r == CFI_MISMATCH) {
        logf_("keeping the stock kernel, %s", w.c_str());
        copy_out(w, why, why_len);
    } else if (r == CFI_SUBSTITUTE) {
        logf_("%s -> native %s (layout %016llx)", mangled, out->key, (unsigned long long)out->layout_hash);
    }
    return r;
}

int cfi_switch_allows(const char* t, const char* family, const char* ty) {
    return Switch::parse(t ? t : "").allows(family ? family : "", ty) ? 1 : 0;
}
int cfi_switch_denies(const char* t, const char* family, const char* ty) {
    return Switch::parse(t ? t : "").denies(family ? family : "", ty) ? 1 : 0;
}
int cfi_switch_is_none(const char* t) { return Switch::parse(t ? t : "").is_none() ? 1 : 0; }

int cfi_demangle(const char* mangled, char* base, size_t base_len, int64_t* values, int* kinds, char* names,
                 size_t names_len, int max_args) {
    if (!mangled) return -1;
    auto m = demangle(mangled);
    if (!m) return -1;
    copy_out(m->base, base, base_len);
    std::string joined;
    int n = (int)m->targs.size();
    for (int i = 0; i < n; i++) {
        if (i < max_args) {
            if (values) values[i] = m->targs[i].value;
            if (kinds) kinds[i] = (int)m->targs[i].kind;
        }
        if (i) joined += "\n";
        joined += m->targs[i].name;
    }
    copy_out(joined, names, names_len);
    return n;
}

uint64_t cfi_layout_hash(const cfi_param* params, int nparams) { return layout_hash(params, nparams); }

int cfi_mmvq_fast_from(const char* text, uint32_t ty, cfi_fast* out) {
    auto f = mmvq_fast_from(text, ty);
    if (!f) return 0;
    if (out) *out = *f;
    return 1;
}
int cfi_mmvq_fast_is_opt_out(const char* text) { return mmvq_fast_is_opt_out(text ? text : "") ? 1 : 0; }
void cfi_mmvq_fast_default(uint32_t ty, cfi_fast* out) {
    if (out) *out = mmvq_fast_default(ty);
}
void cfi_mmvq_key(uint32_t ty, uint32_t ncols, const cfi_fast* fast, uint32_t nwarps, char* out, size_t len) {
    copy_out(mmvq_key(ty, ncols, fast, nwarps), out, len);
}

void cfi_plan_entry_name(const cfi_plan* plan, char* out, size_t len) {
    if (!plan) return;
    char buf[96] = "";
    switch (plan->kernel) {
    case CFI_K_MMVQ:
        if (plan->has_fast)
            snprintf(buf, sizeof buf, "cfi_mmvq_fast_t%u_r%u_w%u_u%u%s", plan->ty, plan->fast.rows, plan->fast.warps,
                     plan->fast.unroll, plan->fast.wide ? "_wide" : "");
        else
            snprintf(buf, sizeof buf, "cfi_mmvq_t%u_c%u_w%u", plan->ty, plan->ncols,
                     plan->nwarps ? plan->nwarps : ggml_mmvq_nwarps(plan->ncols));
        break;
    case CFI_K_QUANTIZE_Q8_1: snprintf(buf, sizeof buf, "cfi_quantize_q8_1"); break;
    case CFI_K_MMQ:
        if (plan->ty == 8)
            snprintf(buf, sizeof buf, "cfi_mmq_q8_0");
        else
            snprintf(buf, sizeof buf, "cfi_mmq_t%u", plan->ty);
        break;
    case CFI_K_QUANTIZE_MMQ: snprintf(buf, sizeof buf, "cfi_quantize_mmq_q8_1_l%u", plan->ty); break;
    case CFI_K_RMS_NORM: snprintf(buf, sizeof buf, "cfi_rms_norm_m%u_a%u", plan->aux & 1, (plan->aux >> 1) & 1); break;
    case CFI_K_RMS_NORM_PLAIN: snprintf(buf, sizeof buf, "cfi_rms_norm_plain"); break;
    case CFI_K_ROPE_NEOX: snprintf(buf, sizeof buf, "cfi_rope_neox_f%u_ff%u", plan->aux & 1, (plan->aux >> 1) & 1); break;
    case CFI_K_SOFT_MAX: snprintf(buf, sizeof buf, "cfi_soft_max_%s", plan->aux ? "f16" : "f32"); break;
    case CFI_K_FATTN: snprintf(buf, sizeof buf, "cfi_fattn_tc_d%u", plan->aux); break;
    default: break;
    }
    copy_out(buf, out, len);
}

int cfi_plan_map_geometry(const cfi_plan* plan, const uint32_t grid[3], const uint32_t block[3], uint32_t grid_out[3],
                          uint32_t block_out[3]) {
    if (!plan || !grid || !block) return 0;
    // kernels whose geometry needs argument values answer through cfi_plan_map_launch
    if (plan->kernel == CFI_K_MMVQ || plan->kernel == CFI_K_MMQ || plan->kernel == CFI_K_ROPE_NEOX) return 0;
    NativeLaunch nl;
    std::vector<uint64_t> vals(nparams_for(plan->kernel, plan->aux), 0);
    if (plan->kernel == CFI_K_QUANTIZE_Q8_1 || plan->kernel == CFI_K_QUANTIZE_MMQ) vals.assign(vals.size(), 0);
    if (!map_launch(*plan, grid, block, vals.data(), (int)vals.size(), nullptr, &nl)) return 0;
    if (grid_out) memcpy(grid_out, nl.grid, sizeof nl.grid);
    if (block_out) memcpy(block_out, nl.block, sizeof nl.block);
    return 1;
}

int cfi_plan_map_launch(const cfi_plan* plan, const uint32_t grid[3], const uint32_t block[3], const uint64_t* vals, int nvals,
                        uint32_t grid_out[3], uint32_t block_out[3]) {
    if (!plan || !grid || !block || (nvals > 0 && !vals)) return 0;
    NativeLaunch nl;
    if (!map_launch(*plan, grid, block, vals, nvals, nullptr, &nl)) return 0;
    if (grid_out) memcpy(grid_out, nl.grid, sizeof nl.grid);
    if (block_out) memcpy(block_out, nl.block, sizeof nl.block);
    return 1;
}

int cfi_plan_extra_word(const cfi_plan* plan, const uint32_t grid[3], uint32_t* word) {
    if (!plan || !grid) return 0;
    if (plan->kernel == CFI_K_MMVQ && plan->ncols == 1) {
        if (word) *word = grid[0];
        return 1;
    }
    if (plan->kernel == CFI_K_ROPE_NEOX) {
        if (word) *word = grid[0];
        return 1;
    }
    return 0;
}

cfi_ctx* cfi_ctx_create(int device, int flags) {
    cfi_ctx* c = new (std::nothrow) cfi_ctx();
    if (!c) return nullptr;
    c->device = device;
    c->flags = flags;
    return c;
}

void cfi_ctx_destroy(cfi_ctx* ctx) {
    if (!ctx) return;
    {
        std::lock_guard<std::mutex> g(ctx->mu);
        flush_deferred(ctx);
    }
    delete ctx;
}

int cfi_ctx_flush(cfi_ctx* ctx) {
    if (!ctx) return (int)cudaErrorInvalidValue;
    std::lock_guard<std::mutex> g(ctx->mu);
    return flush_deferred(ctx);
}

int cfi_subst_launch(cfi_ctx* ctx, const cfi_plan* plan, void* stock_fn, const uint32_t grid[3], const uint32_t block[3],
                     uint32_t shared_bytes, void* stream, void** kernel_params) {
    if (!ctx || !grid || !block) return (int)cudaErrorInvalidValue;
    return launch_to(ctx, plan, stock_fn, grid, block, shared_bytes, stream, kernel_params);
}

int cfi_subst_probe(cfi_ctx* ctx, const cfi_plan* plan, void* stream, char* why, size_t why_len) {
    if (!ctx || !plan) return (int)cudaErrorInvalidValue;
    std::lock_guard<std::mutex> g(ctx->mu);
    std::string w;
    int code = 0;
    ctx->stats.probes_run++;
    int rc;
    if (injected(ctx, CFI_SITE_PROBE, &code)) {
        rc = code;
        w = "injected";
    } else if (ctx->flags & CFI_CTX_FAKE) {
        rc = 0;
    } else {
        rc = probe_validate(*plan, stream, &w);
    }
    if (rc) ctx->stats.probes_failed++;
    copy_out(w, why, why_len);
    return rc;
}

int cfi_ctx_native_state(cfi_ctx* ctx, const char* key) {
    if (!ctx || !key) return 0;
    std::lock_guard<std::mutex> g(ctx->mu);
    auto it = ctx->natives.find(key);
    return it == ctx->natives.end() ? 0 : it->second;
}

void cfi_ctx_stats(cfi_ctx* ctx, cfi_stats* out) {
    if (!ctx || !out) return;
    std::lock_guard<std::mutex> g(ctx->mu);
    *out = ctx->stats;
}

void cfi_ctx_inject(cfi_ctx* ctx, int site, int nth, int code) {
    if (!ctx || site <= 0 || site > 4) return;
    std::lock_guard<std::mutex> g(ctx->mu);
    ctx->inject[site].nth = nth;
    ctx->inject[site].code = code;
    ctx->inject[site].calls = 0;
}

const char* cfi_version(void) { return "cfi_b200 0.1 (sm_100a)"; }

}  // extern "C"
