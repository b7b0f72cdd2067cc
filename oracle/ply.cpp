// ply.cpp - CPU restatement of the splat PLY import / export (test oracle).
//
// TEST INFRASTRUCTURE ONLY: the checker for the GPU PLY path, never part of
// the product.
//
// Follows crates/brush-serde/src/import.rs row by row: parse_ply (:341-502:
// PlyGaussian fields, RGB override via rgb_to_sh, interleave_coeffs :133-144,
// SplatData::into_splats defaults :77-95), parse_compressed_ply (:504-752:
// QuantMeta lerp, QuantSplat decode from quant.rs :4-61, inverse_sigmoid of
// the packed alpha, de_quant_sh ply_gaussian.rs:131-138), and export.rs
// read_splat_data (:84-167). Supports ascii and binary_little_endian input
// (the formats the tests write). Compiled with -ffp-contract=off; ln is the
// shared bsx_logf.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "../include/bsx_fmath.h"

namespace {

struct OProp {
    std::string name;
    std::string type;
    size_t offset;
    size_t size;
};
struct OElem {
    std::string name;
    size_t count;
    std::vector<OProp> props;
    size_t stride;
};

size_t type_size(const std::string& t) {
    if (t == "char" || t == "uchar" || t == "int8" || t == "uint8") return 1;
    if (t == "short" || t == "ushort" || t == "int16" || t == "uint16") return 2;
    if (t == "double" || t == "float64") return 8;
    return 4;
}

// One property value of a row as a double plus its PLY type name.
struct Value {
    double v = 0.0;
    std::string type;
    bool present = false;
};

double decode_binary(const uint8_t* p, const std::string& t) {
    if (t == "char" || t == "int8") return (double)(int8_t)p[0];
    if (t == "uchar" || t == "uint8") return (double)p[0];
    if (t == "short" || t == "int16") { int16_t x; memcpy(&x, p, 2); return x; }
    if (t == "ushort" || t == "uint16") { uint16_t x; memcpy(&x, p, 2); return x; }
    if (t == "int" || t == "int32") { int32_t x; memcpy(&x, p, 4); return x; }
    if (t == "uint" || t == "uint32") { uint32_t x; memcpy(&x, p, 4); return x; }
    if (t == "double" || t == "float64") { double x; memcpy(&x, p, 8); return x; }
    float x;
    memcpy(&x, p, 4);
    return x;
}

struct Ply {
    bool ascii = false;
    std::vector<OElem> elems;
    std::vector<std::vector<std::map<std::string, Value>>> rows;  // per element, per row
};

bool parse(const uint8_t* bytes, size_t len, Ply* ply, std::string* err) {
    size_t pos = 0;
    auto line = [&](std::string* out) {
        size_t e = pos;
        while (e < len && bytes[e] != '\n') ++e;
        if (e >= len) return false;
        out->assign((const char*)bytes + pos, e - pos);
        if (!out->empty() && out->back() == '\r') out->pop_back();
        pos = e + 1;
        return true;
    };
    std::string l;
    if (!line(&l) || l != "ply") { *err = "missing PLY header"; return false; }
    while (line(&l)) {
        std::istringstream ss(l);
        std::string kw;
        ss >> kw;
        if (kw == "format") {
            std::string f;
            ss >> f;
            ply->ascii = f == "ascii";
        } else if (kw == "element") {
            OElem e;
            ss >> e.name >> e.count;
            e.stride = 0;
            ply->elems.push_back(e);
        } else if (kw == "property") {
            OProp p;
            ss >> p.type >> p.name;
            p.size = type_size(p.type);
            p.offset = ply->elems.back().stride;
            ply->elems.back().stride += p.size;
            ply->elems.back().props.push_back(p);
        } else if (kw == "end_header") {
            break;
        }
    }
    ply->rows.resize(ply->elems.size());
    if (ply->ascii) {
        std::string body((const char*)bytes + pos, len - pos);
        std::istringstream ss(body);
        for (size_t k = 0; k < ply->elems.size(); ++k)
            for (size_t r = 0; r < ply->elems[k].count; ++r) {
                std::map<std::string, Value> row;
                for (const OProp& p : ply->elems[k].props) {
                    std::string tok;
                    if (!(ss >> tok)) { *err = "Unexpected EOF while reading PLY data"; return false; }
                    Value v;
                    v.type = p.type;
                    v.present = true;
                    v.v = strtod(tok.c_str(), nullptr);
                    if (p.type == "float" || p.type == "float32") v.v = strtof(tok.c_str(), nullptr);
                    row[p.name] = v;
                }
                ply->rows[k].push_back(row);
            }
    } else {
        for (size_t k = 0; k < ply->elems.size(); ++k)
            for (size_t r = 0; r < ply->elems[k].count; ++r) {
                if (pos + ply->elems[k].stride > len) { *err = "Unexpected EOF while reading PLY data"; return false; }
                std::map<std::string, Value> row;
                for (const OProp& p : ply->elems[k].props) {
                    Value v;
                    v.type = p.type;
                    v.present = true;
                    v.v = decode_binary(bytes + pos + p.offset, p.type);
                    row[p.name] = v;
                }
                pos += ply->elems[k].stride;
                ply->rows[k].push_back(row);
            }
    }
    return true;
}

float as_f32(const Value& v) { return (float)v.v; }
float get(const std::map<std::string, Value>& row, const std::string& name) {
    auto it = row.find(name);
    return it == row.end() ? 0.0f : as_f32(it->second);  // serde default
}
float de_quant(const Value& v) {
    if (v.type == "uchar" || v.type == "uint8") return (float)(uint32_t)v.v / 255.0f;
    if (v.type == "ushort" || v.type == "uint16") return (float)(uint32_t)v.v / 65535.0f;
    return (float)v.v;
}
float channel_to_sh(float c) { return (c - 0.5f) / 0.2820948f; }
float inverse_sigmoid(float x) { return bsx_logf(x / (1.0f - x)); }
float unorm(uint32_t v, uint32_t bits) { return (float)v / (float)((1u << bits) - 1u); }

}  // namespace

extern "C" {

// Decodes a PLY into splat arrays. With null outputs only *n_out / *coeffs_out
// are filled. Returns 0 on success, 1 on a parse error (message in err).
int orc_ply_decode(const uint8_t* bytes, size_t len, uint32_t subsample, uint32_t* n_out, uint32_t* coeffs_out,
                   float* transforms, float* sh, float* opac, char* err, size_t err_len) {
    Ply ply;
    std::string e;
    auto fail = [&](const std::string& m) {
        if (err && err_len) {
            strncpy(err, m.c_str(), err_len - 1);
            err[err_len - 1] = 0;
        }
        return 1;
    };
    if (!parse(bytes, len, &ply, &e)) return fail(e);
    int vi = -1;
    for (size_t k = 0; k < ply.elems.size(); ++k)
        if (ply.elems[k].name == "vertex" && vi < 0) vi = (int)k;
    if (vi < 0) return fail("Unknown format");
    const bool compressed = ply.elems.front().name == "chunk";
    const auto& vrows = ply.rows[vi];
    const OElem& V = ply.elems[vi];
    auto has = [&](const OElem& el, const std::string& n) {
        for (const OProp& p : el.props)
            if (p.name == n) return true;
        return false;
    };
    if (compressed) {
        const auto& chunks = ply.rows[0];
        uint32_t rest = 0;
        if (ply.elems.size() > 2) rest = (uint32_t)ply.elems[2].props.size();
        const uint32_t coeffs = 1 + rest / 3;
        uint32_t n = 0;
        for (size_t r = 0; r < vrows.size(); r += subsample) ++n;
        *n_out = n;
        *coeffs_out = coeffs;
        if (!transforms) return 0;
        uint32_t i = 0;
        for (size_t r = 0; r < vrows.size(); r += subsample, ++i) {
            const auto& q = chunks[r / 256];
            const auto& row = vrows[r];
            const uint32_t pp = (uint32_t)row.at("packed_position").v, pr = (uint32_t)row.at("packed_rotation").v;
            const uint32_t ps = (uint32_t)row.at("packed_scale").v, pc = (uint32_t)row.at("packed_color").v;
            const float mean_raw[3] = {unorm((pp >> 21) & 0x7FF, 11), unorm((pp >> 11) & 0x3FF, 10), unorm(pp & 0x7FF, 11)};
            const float scl_raw[3] = {unorm((ps >> 21) & 0x7FF, 11), unorm((ps >> 11) & 0x3FF, 10), unorm(ps & 0x7FF, 11)};
            const char* ax[3] = {"x", "y", "z"};
            float* t = transforms + (size_t)i * 10;
            for (int k = 0; k < 3; ++k) {
                const float mn = get(q, std::string("min_") + ax[k]), mx = get(q, std::string("max_") + ax[k]);
                t[k] = mean_raw[k] * (mx - mn) + mn;
                const float smn = get(q, std::string("min_scale_") + ax[k]), smx = get(q, std::string("max_scale_") + ax[k]);
                t[7 + k] = scl_raw[k] * (smx - smn) + smn;
            }
            // decode_quat
            const uint32_t largest = (pr >> 30) & 3;
            const float norm = 0.5f * 1.41421356f;
            const float a = (unorm((pr >> 20) & 0x3FF, 10) - 0.5f) / norm;
            const float b = (unorm((pr >> 10) & 0x3FF, 10) - 0.5f) / norm;
            const float c = (unorm(pr & 0x3FF, 10) - 0.5f) / norm;
            float quat[4];
            const float vals[3] = {a, b, c};
            quat[largest] = sqrtf(1.0f - (a * a + b * b + c * c));
            int ind = 0;
            for (uint32_t k = 0; k < 4; ++k)
                if (k != largest) quat[k] = vals[ind++];
            for (int k = 0; k < 4; ++k) t[3 + k] = quat[k];
            const float rgba[4] = {unorm((pc >> 24) & 0xFF, 8), unorm((pc >> 16) & 0xFF, 8), unorm((pc >> 8) & 0xFF, 8),
                                   unorm(pc & 0xFF, 8)};
            opac[i] = inverse_sigmoid(rgba[3]);
            const char* cc[3] = {"r", "g", "b"};
            float* s = sh + (size_t)i * coeffs * 3;
            for (int k = 0; k < 3; ++k) {
                const float mn = get(q, std::string("min_") + cc[k]), mx = get(q, std::string("max_") + cc[k]);
                s[k] = channel_to_sh(rgba[k] * (mx - mn) + mn);
            }
            if (rest) {
                const auto& shrow = ply.rows[2][r];
                std::vector<float> restv(rest);
                for (uint32_t k = 0; k < rest; ++k) {
                    const float v = (float)(uint8_t)(uint32_t)shrow.at("f_rest_" + std::to_string(k)).v / 255.0f;
                    restv[k] = (v - 0.5f) * 8.0f;
                }
                const uint32_t per = rest / 3;
                for (uint32_t k = 0; k < per; ++k)
                    for (uint32_t ch = 0; ch < 3; ++ch) s[3 * (k + 1) + ch] = restv[ch * per + k];
            }
        }
        return 0;
    }
    // standard layout
    uint32_t rest = 0;
    for (const OProp& p : V.props)
        if (p.name.rfind("f_rest_", 0) == 0) ++rest;
    const bool has_dc = has(V, "f_dc_0");
    const bool has_rgb = (has(V, "red") || has(V, "r")) && (has(V, "green") || has(V, "g")) && (has(V, "blue") || has(V, "b"));
    const bool color = has_dc || has_rgb;
    const uint32_t coeffs = color ? 1 + rest / 3 : 1;
    uint32_t n = 0;
    for (size_t r = 0; r < vrows.size(); r += subsample) ++n;
    *n_out = n;
    *coeffs_out = coeffs;
    if (!transforms) return 0;
    const bool has_rot = has(V, "rot_0"), has_scale = has(V, "scale_0");
    uint32_t i = 0;
    for (size_t r = 0; r < vrows.size(); r += subsample, ++i) {
        const auto& row = vrows[r];
        float* t = transforms + (size_t)i * 10;
        t[0] = get(row, "x");
        t[1] = get(row, "y");
        t[2] = get(row, "z");
        if (has_rot)
            for (int k = 0; k < 4; ++k) t[3 + k] = get(row, "rot_" + std::to_string(k));
        else {
            t[3] = 1.0f;
            t[4] = t[5] = t[6] = 0.0f;
        }
        for (int k = 0; k < 3; ++k) t[7 + k] = has_scale ? get(row, "scale_" + std::to_string(k)) : -4.0f;
        opac[i] = get(row, "opacity");  // absent: inverse_sigmoid(0.5) = 0
        float* s = sh + (size_t)i * coeffs * 3;
        if (!color) {
            s[0] = s[1] = s[2] = 0.5f;
            continue;
        }
        float dc[3] = {get(row, "f_dc_0"), get(row, "f_dc_1"), get(row, "f_dc_2")};
        if (has_rgb) {
            auto pick = [&](const char* a, const char* b) { return row.count(a) ? row.at(a) : row.at(b); };
            dc[0] = channel_to_sh(de_quant(pick("red", "r")));
            dc[1] = channel_to_sh(de_quant(pick("green", "g")));
            dc[2] = channel_to_sh(de_quant(pick("blue", "b")));
        }
        // interleave_coeffs: [dc rgb], then per coefficient the three channels
        for (int k = 0; k < 3; ++k) s[k] = dc[k];
        const uint32_t per = rest / 3;
        for (uint32_t k = 0; k < per; ++k)
            for (uint32_t ch = 0; ch < 3; ++ch) s[3 * (k + 1) + ch] = get(row, "f_rest_" + std::to_string(ch * per + k));
    }
    return 0;
}

// Rows of splat_to_ply's vertex element (no header): returns the byte count.
uint64_t orc_ply_encode_rows(const float* transforms, const float* sh, const float* opac, uint32_t n, uint32_t coeffs,
                             uint8_t* out) {
    const uint32_t rest = coeffs - 1;
    size_t o = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const float* t = transforms + (size_t)i * 10;
        const float* s = sh + (size_t)i * coeffs * 3;
        const float r0 = t[3], r1 = t[4], r2 = t[5], r3 = t[6];
        const float rn = fmaxf(sqrtf(r0 * r0 + r1 * r1 + r2 * r2 + r3 * r3), 1e-12f);
        std::vector<float> row = {t[0], t[1], t[2], t[7], t[8], t[9], opac[i], r0 / rn, r1 / rn, r2 / rn, r3 / rn,
                                  s[0], s[1], s[2]};
        for (uint32_t ch = 0; ch < 3; ++ch)
            for (uint32_t k = 1; k <= rest; ++k) row.push_back(s[3 * k + ch]);
        if (out) memcpy(out + o, row.data(), row.size() * 4);
        o += row.size() * 4;
    }
    return o;
}

}  // extern "C"
