// ply.cu - splat PLY import and export (brush-serde).
//
// Restates crates/brush-serde/src/import.rs (stream_splat_from_ply :180-296,
// parse_ply :341-502, parse_compressed_ply :504-752, validate_sh_rest_properties
// :306-333, interleave_coeffs :133-144), quant.rs (:4-61) and export.rs
// (read_splat_data :84-167, splat_to_ply :170-191).
//
// B200 design: the host only parses the header (a few hundred bytes) and,
// for ASCII or big-endian files, rewrites the rows as little-endian binary.
// The row blocks go to the GPU in one copy each, and one thread per output
// splat decodes its row straight into the splat tensor layout in HBM
// (transforms [N,10], sh [N,C,3] coefficient-major, raw opacities [N]):
// typed field reads, the RGB-to-SH and logit conversions, the SH
// re-interleave from the file's channel-major order, the default values of
// absent fields and, for the SuperSplat compressed format, the dequantisation
// against each 256-row chunk's bounds. Export runs the inverse: one thread
// per splat writes its little-endian row (quaternion normalised), and the
// host prepends the header.
//
// Arithmetic follows the reference's expressions in the same order (this
// file is compiled without contraction), with bsx_logf for ln, so the CPU
// restatement in the test oracle reproduces every output bit.
#include <algorithm>
#include <cerrno>
#include <charconv>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "common.cuh"

namespace bsx {

namespace {

enum PlyType : int32_t { kI8 = 0, kU8, kI16, kU16, kI32, kU32, kF32, kF64 };
constexpr uint32_t kTypeSize[8] = {1, 1, 2, 2, 4, 4, 4, 8};
constexpr float kShC0 = 0.2820948f;  // SH_C0 (crates/brush-render/src/shaders.rs:6)
constexpr uint32_t kSplatsPerChunk = 256;
constexpr int kMaxRest = 72;

struct Field {
    int32_t offset = -1;  // byte offset in the row, -1 when absent
    int32_t type = kF32;
};

struct Prop {
    std::string name;
    int32_t type = kF32;
    uint32_t offset = 0;
    bool list = false;
};

struct Elem {
    std::string name;
    uint64_t count = 0;
    std::vector<Prop> props;
    uint32_t stride = 0;
    const Prop* find(const std::string& n) const {
        for (const Prop& p : props)
            if (p.name == n) return &p;
        return nullptr;
    }
};

bool parse_type(const std::string& t, int32_t* out) {
    static const char* names[][2] = {{"char", "int8"},   {"uchar", "uint8"},   {"short", "int16"},
                                     {"ushort", "uint16"}, {"int", "int32"},     {"uint", "uint32"},
                                     {"float", "float32"}, {"double", "float64"}};
    for (int i = 0; i < 8; ++i)
        if (t == names[i][0] || t == names[i][1]) {
            *out = i;
            return true;
        }
    return false;
}

std::string lower(std::string s) {
    for (char& c : s) c = (char)tolower((unsigned char)c);
    return s;
}

std::string trim(const std::string& s) {
    size_t a = s.find_first_not_of(" \t\r\n"), b = s.find_last_not_of(" \t\r\n");
    return a == std::string::npos ? std::string() : s.substr(a, b - a + 1);
}

Field field_of(const Elem& e, const char* name, const char* alias = nullptr) {
    const Prop* p = e.find(name);
    if (!p && alias) p = e.find(alias);
    Field f;
    if (p) {
        f.offset = (int32_t)p->offset;
        f.type = p->type;
    }
    return f;
}

// ---- device side ---------------------------------------------------------

__device__ __forceinline__ uint32_t load_bytes(const uint8_t* p, uint32_t n) {
    uint32_t v = 0;
    for (uint32_t i = 0; i < n; ++i) v |= (uint32_t)p[i] << (8 * i);
    return v;
}

// Numeric field as f32, serde's primitive conversion ("as" casts). 4-byte
// fields at 4-byte aligned offsets of 4-byte aligned rows (the usual all-float
// file) take one word load.
__device__ __forceinline__ float read_num(const uint8_t* row, Field f) {
    const uint8_t* p = row + f.offset;
    if (f.type == kF32 && !(reinterpret_cast<uintptr_t>(p) & 3u)) return __ldg(reinterpret_cast<const float*>(p));
    switch (f.type) {
        case kI8: return (float)(int8_t)p[0];
        case kU8: return (float)p[0];
        case kI16: return (float)(int16_t)load_bytes(p, 2);
        case kU16: return (float)(uint16_t)load_bytes(p, 2);
        case kI32: return (float)(int32_t)load_bytes(p, 4);
        case kU32: return (float)load_bytes(p, 4);
        case kF32: return __uint_as_float(load_bytes(p, 4));
        default: {
            const uint64_t lo = load_bytes(p, 4), hi = load_bytes(p + 4, 4);
            return (float)__longlong_as_double((long long)(lo | (hi << 32)));
        }
    }
}

// Colour override (import.rs PlyGaussian red/green/blue, de_quant): u8 / 255,
// u16 / 65535, f32 as is (other types are rejected on the host).
__device__ __forceinline__ float read_color(const uint8_t* row, Field f) {
    const uint8_t* p = row + f.offset;
    if (f.type == kU8) return (float)p[0] / 255.0f;
    if (f.type == kU16) return (float)(uint16_t)load_bytes(p, 2) / 65535.0f;
    return __uint_as_float(load_bytes(p, 4));
}

__device__ __forceinline__ float read_or(const uint8_t* row, Field f, float dflt) {
    return f.offset >= 0 ? read_num(row, f) : dflt;
}

// Integer field as u32 (the packed words and quantised SH of the compressed layout).
__device__ __forceinline__ uint32_t read_u32(const uint8_t* row, Field f) {
    const uint32_t size = (f.type == kI8 || f.type == kU8) ? 1u : (f.type == kI16 || f.type == kU16) ? 2u : 4u;
    return load_bytes(row + f.offset, size);
}

__device__ __forceinline__ float channel_to_sh(float c) { return (c - 0.5f) / kShC0; }
__device__ __forceinline__ float inverse_sigmoid(float x) { return bsx_logf(x / (1.0f - x)); }
__device__ __forceinline__ float unpack_unorm(uint32_t v, uint32_t bits) {
    return (float)v / (float)((1u << bits) - 1u);
}

struct StdArgs {
    const uint8_t* rows;
    uint64_t stride;
    uint32_t n_out, subsample, coeffs, rest;  // rest: f_rest properties in the file (0, 9, 24, 45, 72)
    int32_t color;                            // 0 none, 1 f_dc, 2 rgb override
    Field xyz[3], scale[3], rot[4], opacity, dc[3], rgb[3];
    Field f_rest[kMaxRest];
    float* transforms;
    float* sh;
    float* opac;
};

__global__ void __launch_bounds__(256) ply_decode_kernel(const __grid_constant__ StdArgs a) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n_out) return;
    const uint8_t* row = a.rows + (uint64_t)i * a.subsample * a.stride;
    float* t = a.transforms + (size_t)i * 10;
    for (int k = 0; k < 3; ++k) t[k] = read_num(row, a.xyz[k]);
    // rot_0 / scale_0 decide whether the group is present (import.rs:408-418);
    // a present group's missing members read 0 (serde defaults); absent groups
    // take the Splats defaults (SplatData::into_splats, import.rs:77-95)
    if (a.rot[0].offset >= 0)
        for (int k = 0; k < 4; ++k) t[3 + k] = read_or(row, a.rot[k], 0.0f);
    else {
        t[3] = 1.0f;
        t[4] = t[5] = t[6] = 0.0f;
    }
    for (int k = 0; k < 3; ++k) t[7 + k] = a.scale[0].offset >= 0 ? read_or(row, a.scale[k], 0.0f) : -4.0f;
    a.opac[i] = read_or(row, a.opacity, 0.0f);  // default inverse_sigmoid(0.5) = 0
    float* s = a.sh + (size_t)i * a.coeffs * 3;
    if (a.color == 0) {
        s[0] = s[1] = s[2] = 0.5f;
        return;
    }
    for (int c = 0; c < 3; ++c)
        s[c] = a.color == 2 ? channel_to_sh(read_color(row, a.rgb[c])) : read_num(row, a.dc[c]);
    // file order f_rest_{channel * per + k}, splat order [coefficient][channel]
    const uint32_t per = a.rest / 3;
    for (uint32_t k = 0; k < per; ++k)
        for (int c = 0; c < 3; ++c) s[3 * (k + 1) + c] = read_num(row, a.f_rest[c * per + k]);
}

struct CompArgs {
    const uint8_t* chunks;
    uint64_t chunk_stride;
    Field bounds[18];  // min_x max_x min_y max_y min_z max_z, scales, r g b
    const uint8_t* verts;
    uint64_t vert_stride;
    Field packed[4];   // position, rotation, scale, color
    const uint8_t* shs;
    uint64_t sh_stride;
    Field f_rest[kMaxRest];
    uint32_t rest, n_out, subsample, coeffs;
    float* transforms;
    float* sh;
    float* opac;
};

// decode_quat (quant.rs:38-61): smallest-three 2-10-10-10, stored (w, x, y, z).
__device__ __forceinline__ void decode_quat(uint32_t v, float q[4]) {
    const uint32_t largest = (v >> 30) & 0x3u;
    const float norm = 0.5f * 1.41421356f;
    const float a = (unpack_unorm((v >> 20) & 0x3FFu, 10) - 0.5f) / norm;
    const float b = (unpack_unorm((v >> 10) & 0x3FFu, 10) - 0.5f) / norm;
    const float c = (unpack_unorm(v & 0x3FFu, 10) - 0.5f) / norm;
    const float vals[3] = {a, b, c};
    float quat[4];
    quat[largest] = sqrtf(1.0f - ((a * a + b * b) + c * c));
    int ind = 0;
    for (uint32_t k = 0; k < 4; ++k)
        if (k != largest) quat[k] = vals[ind++];
    for (int k = 0; k < 4; ++k) q[k] = quat[k];
}

__global__ void __launch_bounds__(256) ply_decode_compressed_kernel(const __grid_constant__ CompArgs a) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n_out) return;
    const uint64_t r = (uint64_t)i * a.subsample;
    const uint8_t* chunk = a.chunks + (r / kSplatsPerChunk) * a.chunk_stride;
    const uint8_t* vert = a.verts + r * a.vert_stride;
    float bnd[18];
    for (int k = 0; k < 18; ++k) bnd[k] = read_num(chunk, a.bounds[k]);
    const uint32_t pos = read_u32(vert, a.packed[0]), rot = read_u32(vert, a.packed[1]);
    const uint32_t scl = read_u32(vert, a.packed[2]), col = read_u32(vert, a.packed[3]);
    // decode_vec_11_10_11, then raw * (max - min) + min (QuantMeta::mean / scale)
    const float p3[3] = {unpack_unorm((pos >> 21) & 0x7FFu, 11), unpack_unorm((pos >> 11) & 0x3FFu, 10),
                         unpack_unorm(pos & 0x7FFu, 11)};
    const float s3[3] = {unpack_unorm((scl >> 21) & 0x7FFu, 11), unpack_unorm((scl >> 11) & 0x3FFu, 10),
                         unpack_unorm(scl & 0x7FFu, 11)};
    float* t = a.transforms + (size_t)i * 10;
    for (int k = 0; k < 3; ++k) {
        t[k] = p3[k] * (bnd[2 * k + 1] - bnd[2 * k]) + bnd[2 * k];
        t[7 + k] = s3[k] * (bnd[6 + 2 * k + 1] - bnd[6 + 2 * k]) + bnd[6 + 2 * k];
    }
    float q[4];
    decode_quat(rot, q);
    for (int k = 0; k < 4; ++k) t[3 + k] = q[k];
    // decode_vec_8_8_8_8: x = bits 24-31 ... w = bits 0-7; opacity is post-activation
    const float rgba[4] = {unpack_unorm((col >> 24) & 0xFFu, 8), unpack_unorm((col >> 16) & 0xFFu, 8),
                           unpack_unorm((col >> 8) & 0xFFu, 8), unpack_unorm(col & 0xFFu, 8)};
    a.opac[i] = inverse_sigmoid(rgba[3]);
    float* s = a.sh + (size_t)i * a.coeffs * 3;
    for (int c = 0; c < 3; ++c)
        s[c] = channel_to_sh(rgba[c] * (bnd[12 + 2 * c + 1] - bnd[12 + 2 * c]) + bnd[12 + 2 * c]);
    if (!a.rest) return;
    const uint8_t* shr = a.shs + r * a.sh_stride;
    const uint32_t per = a.rest / 3;
    for (uint32_t k = 0; k < per; ++k)
        for (int c = 0; c < 3; ++c) {
            // de_quant_sh (ply_gaussian.rs:131-138): (v / 255 - 0.5) * 8
            const float v = (float)(uint8_t)read_u32(shr, a.f_rest[c * per + k]) / 255.0f;
            s[3 * (k + 1) + c] = (v - 0.5f) * 8.0f;
        }
}

struct EncArgs {
    const float* transforms;
    const float* sh;
    const float* opac;
    uint32_t n, coeffs;
    uint8_t* out;  // rows of (14 + 3 (coeffs - 1)) little-endian f32
};

// Rows are whole 4-byte words and the staging buffer is aligned: word stores
// (the device is little-endian like the file).
__device__ __forceinline__ void put_f32(uint8_t* p, float v) { *reinterpret_cast<float*>(p) = v; }

// read_splat_data (export.rs:84-167): x y z, scale_0..2, opacity, rot_0..3
// normalised by max(|q|, 1e-12), f_dc_0..2, f_rest_{channel * rest + k}.
__global__ void __launch_bounds__(256) ply_encode_kernel(const __grid_constant__ EncArgs a) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    const uint32_t rest = a.coeffs - 1, fields = 14 + 3 * rest;
    uint8_t* row = a.out + (size_t)i * fields * 4;
    const float* t = a.transforms + (size_t)i * 10;
    const float* s = a.sh + (size_t)i * a.coeffs * 3;
    const float r0 = t[3], r1 = t[4], r2 = t[5], r3 = t[6];
    const float rn = fmaxf(sqrtf(((r0 * r0 + r1 * r1) + r2 * r2) + r3 * r3), 1e-12f);
    const float v[14] = {t[0], t[1], t[2], t[7], t[8], t[9], a.opac[i], r0 / rn, r1 / rn, r2 / rn, r3 / rn,
                         s[0], s[1], s[2]};
    for (int k = 0; k < 14; ++k) put_f32(row + 4 * k, v[k]);
    for (int c = 0; c < 3; ++c)
        for (uint32_t k = 0; k < rest; ++k) put_f32(row + 4 * (14 + c * rest + k), s[3 * (k + 1) + c]);
}

}  // namespace
}  // namespace bsx

// ---- host side: header parse, row blocks, C ABI ---------------------------

struct bsx_ply_file {
    bsx_ply_info info{};
    bool compressed = false;
    std::vector<bsx::Elem> elems;
    // little-endian row blocks: either views into the caller's bytes or owned copies
    std::vector<const uint8_t*> block;
    std::vector<std::vector<uint8_t>> owned;
    int color = 0;
    uint32_t rest = 0;
    int vertex = -1, chunk = -1, sh = -1;
    std::string error;
};

namespace {

using bsx::Elem;
using bsx::Prop;

bsx_status ply_fail(bsx_ply_file* f, const std::string& m, char* err, size_t err_len) {
    if (err && err_len) {
        std::strncpy(err, m.c_str(), err_len - 1);
        err[err_len - 1] = 0;
    }
    (void)f;
    return BSX_ERR_FORMAT;
}

// validate_sh_rest_properties (import.rs:306-333)
bool validate_rest(const Elem& e, bool all_props, uint32_t* count, std::string* msg) {
    std::vector<uint32_t> idx;
    for (const Prop& p : e.props) {
        const bool rest = p.name.rfind("f_rest_", 0) == 0;
        if (!rest && !all_props) continue;
        const char* s = p.name.c_str() + 7;
        uint32_t v = 0;
        auto r = std::from_chars(s, p.name.c_str() + p.name.size(), v);
        if (!rest || r.ec != std::errc() || r.ptr != p.name.c_str() + p.name.size() || p.name.size() == 7) {
            *msg = "Invalid SH property name: " + p.name;
            return false;
        }
        idx.push_back(v);
    }
    std::sort(idx.begin(), idx.end());
    for (size_t k = 0; k < idx.size(); ++k)
        if (idx[k] != k) {
            *msg = "SH rest properties must be contiguous from f_rest_0";
            return false;
        }
    if (!(idx.size() == 0 || idx.size() == 9 || idx.size() == 24 || idx.size() == 45 || idx.size() == 72)) {
        *msg = "Unsupported SH rest property count: " + std::to_string(idx.size());
        return false;
    }
    *count = (uint32_t)idx.size();
    return true;
}

bool parse_float(const std::string& s, float* out) {
    const char* b = s.c_str();
    char* e = nullptr;
    errno = 0;
    const float v = std::strtof(b, &e);
    if (e == b || *e) return false;
    *out = v;
    return true;
}

// Up axis and render mode from the header comments, last one wins (import.rs:205-245).
void parse_comments(const std::vector<std::string>& comments, bsx_ply_info* info) {
    for (const std::string& c : comments) {
        const std::string s = bsx::lower(c);
        const std::string ax = "vertical axis: ", rm = "splatrendermode: ";
        if (s.rfind(ax, 0) == 0) {
            const std::string v = bsx::trim(s.substr(ax.size()));
            float u[3] = {0, 0, 0};
            bool ok = true;
            if (v == "x") u[0] = 1.0f;
            else if (v == "y") u[1] = -1.0f;
            else if (v == "z") u[2] = -1.0f;
            else {
                std::vector<float> parts;
                std::string tok;
                for (size_t k = 0; k <= v.size(); ++k) {
                    const char ch = k < v.size() ? v[k] : ' ';
                    if (ch == ',' || isspace((unsigned char)ch) || ch == '[' || ch == ']') {
                        float x;
                        if (!tok.empty() && parse_float(tok, &x)) parts.push_back(x);
                        tok.clear();
                    } else {
                        tok.push_back(ch);
                    }
                }
                ok = parts.size() == 3;
                if (ok)
                    for (int k = 0; k < 3; ++k) u[k] = parts[k];
            }
            if (ok) {
                info->has_up_axis = 1;
                for (int k = 0; k < 3; ++k) info->up_axis[k] = u[k];
            }
        } else if (s.rfind(rm, 0) == 0) {
            const std::string v = bsx::trim(s.substr(rm.size()));
            if (v == "mip") info->render_mode = 1;
            else if (v == "default") info->render_mode = 0;
        }
    }
}

template <typename T>
void put_le(uint8_t* p, T v) {
    std::memcpy(p, &v, sizeof v);  // the host is little-endian
}

// One ASCII token as a typed little-endian value.
bool ascii_value(const std::string& tok, int32_t type, uint8_t* dst) {
    const char* b = tok.c_str();
    char* e = nullptr;
    if (type == bsx::kF32 || type == bsx::kF64) {
        const double d = std::strtod(b, &e);
        if (e == b || *e) return false;
        if (type == bsx::kF32) put_le<float>(dst, std::strtof(b, nullptr));
        else put_le<double>(dst, d);
        return true;
    }
    const long long v = std::strtoll(b, &e, 10);
    if (e == b || *e) return false;
    switch (type) {
        case bsx::kI8: put_le<int8_t>(dst, (int8_t)v); break;
        case bsx::kU8: put_le<uint8_t>(dst, (uint8_t)v); break;
        case bsx::kI16: put_le<int16_t>(dst, (int16_t)v); break;
        case bsx::kU16: put_le<uint16_t>(dst, (uint16_t)v); break;
        case bsx::kI32: put_le<int32_t>(dst, (int32_t)v); break;
        default: put_le<uint32_t>(dst, (uint32_t)v); break;
    }
    return true;
}

}  // namespace

extern "C" {

bsx_status bsx_ply_parse(const uint8_t* bytes, size_t len, uint32_t subsample, bsx_ply_file** out, bsx_ply_info* info,
                         char* err, size_t err_len) {
    if (!out || !info || (len && !bytes)) return BSX_ERR_INVALID_ARG;
    *out = nullptr;
    std::unique_ptr<bsx_ply_file> f(new bsx_ply_file());
    bsx_ply_file* F = f.get();
    F->info.render_mode = -1;
    if (subsample == 0) return ply_fail(F, "subsample_points must be greater than zero", err, err_len);
    if (len == 0) return ply_fail(F, "Unexpected EOF while reading PLY data", err, err_len);

    // ---- header
    size_t pos = 0;
    auto next_line = [&](std::string* line) -> bool {
        if (pos >= len) return false;
        const void* nl = std::memchr(bytes + pos, '\n', len - pos);
        if (!nl) return false;
        const size_t e = (size_t)(static_cast<const uint8_t*>(nl) - (bytes + pos));
        line->assign(reinterpret_cast<const char*>(bytes) + pos, e);
        if (!line->empty() && line->back() == '\r') line->pop_back();
        pos += e + 1;
        return true;
    };
    std::string line;
    if (!next_line(&line) || bsx::trim(line) != "ply") return ply_fail(F, "missing PLY header", err, err_len);
    int format = -1;
    std::vector<std::string> comments;
    bool done = false;
    while (next_line(&line)) {
        std::istringstream ss(line);
        std::string kw;
        ss >> kw;
        if (kw == "format") {
            std::string fm;
            ss >> fm;
            format = fm == "ascii" ? 0 : fm == "binary_little_endian" ? 1 : fm == "binary_big_endian" ? 2 : -2;
        } else if (kw == "comment") {
            std::string rest = line.size() > 8 ? line.substr(8) : std::string();
            comments.push_back(rest);
        } else if (kw == "obj_info" || kw.empty()) {
        } else if (kw == "element") {
            Elem e;
            ss >> e.name >> e.count;
            if (ss.fail()) return ply_fail(F, "missing PLY header", err, err_len);
            F->elems.push_back(e);
        } else if (kw == "property") {
            if (F->elems.empty()) return ply_fail(F, "missing PLY header", err, err_len);
            Prop p;
            std::string t;
            ss >> t;
            if (t == "list") {
                std::string ct, it;
                ss >> ct >> it >> p.name;
                p.list = true;
            } else {
                if (!bsx::parse_type(t, &p.type)) return ply_fail(F, "Unknown PLY property type: " + t, err, err_len);
                ss >> p.name;
            }
            F->elems.back().props.push_back(p);
        } else if (kw == "end_header") {
            done = true;
            break;
        }
    }
    if (!done || format < 0) return ply_fail(F, "missing PLY header", err, err_len);
    for (Elem& e : F->elems) {
        uint32_t off = 0;
        for (Prop& p : e.props) {
            p.offset = off;
            off += p.list ? 0 : bsx::kTypeSize[p.type];
        }
        e.stride = off;
    }
    parse_comments(comments, &F->info);

    // ---- format detection (import.rs:250-264)
    for (size_t k = 0; k < F->elems.size(); ++k) {
        if (F->elems[k].name == "vertex" && F->vertex < 0) F->vertex = (int)k;
        if (F->elems[k].name == "chunk" && F->chunk < 0) F->chunk = (int)k;
        if (F->elems[k].name == "sh" && F->sh < 0) F->sh = (int)k;
    }
    if (F->vertex < 0) return ply_fail(F, "Unknown format", err, err_len);
    F->compressed = F->elems.front().name == "chunk";
    const Elem& V = F->elems[F->vertex];
    if (V.count == 0) return ply_fail(F, "PLY contains no vertices", err, err_len);
    if (V.count >= (1ull << 31)) return ply_fail(F, "PLY vertex count out of range", err, err_len);
    for (const Elem& e : F->elems)
        for (const Prop& p : e.props)
            if (p.list && (&e == &V || e.name == "chunk" || e.name == "sh"))
                return ply_fail(F, "PLY list properties are not supported in splat elements", err, err_len);

    std::string msg;
    if (F->compressed) {
        const uint64_t need = (V.count + bsx::kSplatsPerChunk - 1) / bsx::kSplatsPerChunk;
        if (F->elems.front().count < need)
            return ply_fail(F, "Compressed PLY has " + std::to_string(F->elems.front().count) +
                                   " chunk rows but needs at least " + std::to_string(need) + " for " +
                                   std::to_string(V.count) + " vertices", err, err_len);
        if (F->vertex != 1) return ply_fail(F, "Unknown format", err, err_len);
        if (F->elems.size() > 2) {
            const Elem& S = F->elems[2];
            if (S.name != "sh" || S.count != V.count)
                return ply_fail(F, "Invalid compressed PLY SH element: expected " + std::to_string(V.count) + " rows",
                                err, err_len);
            if (!validate_rest(S, true, &F->rest, &msg)) return ply_fail(F, msg, err, err_len);
            for (const Prop& p : S.props)
                if (p.type == bsx::kF32 || p.type == bsx::kF64)
                    return ply_fail(F, "Compressed PLY SH values must be integers", err, err_len);
        }
        static const char* bnames[18] = {"min_x", "max_x", "min_y", "max_y", "min_z", "max_z",
                                         "min_scale_x", "max_scale_x", "min_scale_y", "max_scale_y",
                                         "min_scale_z", "max_scale_z", "min_r", "max_r", "min_g", "max_g",
                                         "min_b", "max_b"};
        for (const char* b : bnames)
            if (!F->elems.front().find(b))
                return ply_fail(F, std::string("missing field `") + b + "`", err, err_len);
        static const char* pnames[4] = {"packed_position", "packed_rotation", "packed_scale", "packed_color"};
        for (const char* b : pnames) {
            const Prop* p = V.find(b);
            if (!p) return ply_fail(F, std::string("missing field `") + b + "`", err, err_len);
            if (p->type == bsx::kF32 || p->type == bsx::kF64)
                return ply_fail(F, std::string("invalid type for `") + b + "`", err, err_len);
        }
        F->color = 1;
        F->info.sh_coeffs = 1 + F->rest / 3;
    } else {
        if (!validate_rest(V, false, &F->rest, &msg)) return ply_fail(F, msg, err, err_len);
        int dc = 0;
        for (const char* n : {"f_dc_0", "f_dc_1", "f_dc_2"}) dc += V.find(n) ? 1 : 0;
        int rgb[3] = {0, 0, 0};
        const char* cn[3][2] = {{"r", "red"}, {"g", "green"}, {"b", "blue"}};
        for (int c = 0; c < 3; ++c)
            for (const Prop& p : V.props) rgb[c] += (p.name == cn[c][0] || p.name == cn[c][1]) ? 1 : 0;
        const bool has_rgb = rgb[0] == 1 && rgb[1] == 1 && rgb[2] == 1;
        if (dc != 0 && dc != 3) return ply_fail(F, "PLY SH colors require f_dc_0, f_dc_1, and f_dc_2", err, err_len);
        if ((rgb[0] || rgb[1] || rgb[2]) && !has_rgb)
            return ply_fail(F, "PLY RGB colors require exactly one red, green, and blue property", err, err_len);
        const bool has_color = dc == 3 || has_rgb;
        if (F->rest > 0 && !has_color)
            return ply_fail(F, "PLY SH rest properties require a complete DC or RGB color", err, err_len);
        if (has_rgb)
            for (int c = 0; c < 3; ++c) {
                const bsx::Field fc = bsx::field_of(V, cn[c][1], cn[c][0]);
                if (!(fc.type == bsx::kU8 || fc.type == bsx::kU16 || fc.type == bsx::kF32))
                    return ply_fail(F, "PLY colour properties must be uchar, ushort or float", err, err_len);
            }
        for (const char* n : {"x", "y", "z"})
            if (!V.find(n)) return ply_fail(F, std::string("missing field `") + n + "`", err, err_len);
        F->color = has_rgb ? 2 : has_color ? 1 : 0;
        F->info.sh_coeffs = has_color ? 1 + F->rest / 3 : 1;
    }
    F->info.compressed = F->compressed ? 1 : 0;
    F->info.total_rows = (uint32_t)V.count;
    F->info.num_splats = (uint32_t)((V.count + subsample - 1) / subsample);
    F->info.subsample = subsample;

    // ---- row blocks (little-endian binary), in element order
    F->block.assign(F->elems.size(), nullptr);
    F->owned.resize(F->elems.size());
    if (format == 0) {
        // ASCII: whitespace-separated tokens, one per property, rows in order
        const char* p = reinterpret_cast<const char*>(bytes) + pos;
        const char* end = reinterpret_cast<const char*>(bytes) + len;
        auto token = [&](std::string* t) -> bool {
            while (p < end && isspace((unsigned char)*p)) ++p;
            const char* b = p;
            while (p < end && !isspace((unsigned char)*p)) ++p;
            t->assign(b, p);
            return p > b;
        };
        std::string tok;
        for (size_t k = 0; k < F->elems.size(); ++k) {
            const Elem& e = F->elems[k];
            const bool needed = (int)k == F->vertex || (int)k == F->chunk || (int)k == F->sh;
            if (needed) F->owned[k].resize(e.count * e.stride);
            for (uint64_t r = 0; r < e.count; ++r)
                for (const Prop& pr : e.props) {
                    if (pr.list) {
                        std::string cnt;
                        if (!token(&cnt)) return ply_fail(F, "Unexpected EOF while reading PLY data", err, err_len);
                        const long nlist = std::strtol(cnt.c_str(), nullptr, 10);
                        for (long q = 0; q < nlist; ++q)
                            if (!token(&tok)) return ply_fail(F, "Unexpected EOF while reading PLY data", err, err_len);
                        continue;
                    }
                    if (!token(&tok)) return ply_fail(F, "Unexpected EOF while reading PLY data", err, err_len);
                    if (needed && !ascii_value(tok, pr.type, F->owned[k].data() + r * e.stride + pr.offset))
                        return ply_fail(F, "Invalid PLY value: " + tok, err, err_len);
                }
            if (needed) F->block[k] = F->owned[k].data();
        }
    } else {
        size_t off = pos;
        for (size_t k = 0; k < F->elems.size(); ++k) {
            const Elem& e = F->elems[k];
            bool has_list = false;
            for (const Prop& pr : e.props) has_list |= pr.list;
            if (has_list) {
                if ((int)k < std::max(F->vertex, std::max(F->chunk, F->sh)))
                    return ply_fail(F, "PLY list elements before the splat rows are not supported", err, err_len);
                break;
            }
            const uint64_t bytes_k = e.count * (uint64_t)e.stride;
            if (off + bytes_k > len) {
                const bool needed = (int)k == F->vertex || (int)k == F->chunk || (int)k == F->sh;
                if (needed) return ply_fail(F, "Unexpected EOF while reading PLY data", err, err_len);
                break;
            }
            if (format == 1) {
                F->block[k] = bytes + off;
            } else {  // big-endian: swap each field
                F->owned[k].assign(bytes + off, bytes + off + bytes_k);
                for (uint64_t r = 0; r < e.count; ++r)
                    for (const Prop& pr : e.props) {
                        uint8_t* q = F->owned[k].data() + r * e.stride + pr.offset;
                        std::reverse(q, q + bsx::kTypeSize[pr.type]);
                    }
                F->block[k] = F->owned[k].data();
            }
            off += bytes_k;
        }
    }
    *info = F->info;
    *out = f.release();
    return BSX_OK;
}

void bsx_ply_free(bsx_ply_file* f) { delete f; }

bsx_status bsx_ply_load(bsx_ctx* ctx, const bsx_ply_file* f, float* d_transforms, float* d_sh, float* d_raw_opac) {
    using namespace bsx;
    if (!ctx || !f || !d_transforms || !d_sh || !d_raw_opac) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    const uint32_t n = f->info.num_splats;
    // Copy the needed row blocks to the device (stream-ordered scratch).
    std::vector<uint8_t*> dev(f->elems.size(), nullptr);
    auto release_all = [&]() {
        for (uint8_t* p : dev)
            if (p) cudaFreeAsync(p, ctx->stream);
    };
    for (size_t k = 0; k < f->elems.size(); ++k) {
        if (!f->block[k]) continue;
        const size_t bytes = f->elems[k].count * (size_t)f->elems[k].stride;
        if (!bytes) continue;
        bsx_status s = check_cuda(ctx, cudaMallocAsync((void**)&dev[k], bytes, ctx->stream), "ply staging");
        if (s == BSX_OK)
            s = check_cuda(ctx, cudaMemcpyAsync(dev[k], f->block[k], bytes, cudaMemcpyHostToDevice, ctx->stream),
                           "ply upload");
        if (s != BSX_OK) {
            release_all();
            return s;
        }
    }
    const uint32_t blocks = (n + 255) / 256;
    bsx_status s = BSX_OK;
    if (!f->compressed) {
        const Elem& V = f->elems[f->vertex];
        StdArgs a{};
        a.rows = dev[f->vertex];
        a.stride = V.stride;
        a.n_out = n;
        a.subsample = f->info.subsample;
        a.coeffs = f->info.sh_coeffs;
        a.rest = f->rest;
        a.color = f->color;
        const char* xyz[3] = {"x", "y", "z"};
        for (int k = 0; k < 3; ++k) a.xyz[k] = field_of(V, xyz[k]);
        for (int k = 0; k < 3; ++k) a.scale[k] = field_of(V, ("scale_" + std::to_string(k)).c_str());
        for (int k = 0; k < 4; ++k) a.rot[k] = field_of(V, ("rot_" + std::to_string(k)).c_str());
        a.opacity = field_of(V, "opacity");
        for (int k = 0; k < 3; ++k) a.dc[k] = field_of(V, ("f_dc_" + std::to_string(k)).c_str());
        a.rgb[0] = field_of(V, "red", "r");
        a.rgb[1] = field_of(V, "green", "g");
        a.rgb[2] = field_of(V, "blue", "b");
        for (uint32_t k = 0; k < f->rest; ++k) a.f_rest[k] = field_of(V, ("f_rest_" + std::to_string(k)).c_str());
        a.transforms = d_transforms;
        a.sh = d_sh;
        a.opac = d_raw_opac;
        if (n) {
            prof_begin(ctx);
            ply_decode_kernel<<<blocks, 256, 0, ctx->stream>>>(a);
            s = post_launch(ctx, "ply_decode_kernel");
        }
    } else {
        const Elem& Cc = f->elems[f->chunk];
        const Elem& V = f->elems[f->vertex];
        CompArgs a{};
        a.chunks = dev[f->chunk];
        a.chunk_stride = Cc.stride;
        static const char* bnames[18] = {"min_x", "max_x", "min_y", "max_y", "min_z", "max_z",
                                         "min_scale_x", "max_scale_x", "min_scale_y", "max_scale_y",
                                         "min_scale_z", "max_scale_z", "min_r", "max_r", "min_g", "max_g",
                                         "min_b", "max_b"};
        for (int k = 0; k < 18; ++k) a.bounds[k] = field_of(Cc, bnames[k]);
        a.verts = dev[f->vertex];
        a.vert_stride = V.stride;
        a.packed[0] = field_of(V, "packed_position");
        a.packed[1] = field_of(V, "packed_rotation");
        a.packed[2] = field_of(V, "packed_scale");
        a.packed[3] = field_of(V, "packed_color");
        if (f->rest) {
            const Elem& S = f->elems[f->sh];
            a.shs = dev[f->sh];
            a.sh_stride = S.stride;
            for (uint32_t k = 0; k < f->rest; ++k) a.f_rest[k] = field_of(S, ("f_rest_" + std::to_string(k)).c_str());
        }
        a.rest = f->rest;
        a.n_out = n;
        a.subsample = f->info.subsample;
        a.coeffs = f->info.sh_coeffs;
        a.transforms = d_transforms;
        a.sh = d_sh;
        a.opac = d_raw_opac;
        if (n) {
            prof_begin(ctx);
            ply_decode_compressed_kernel<<<blocks, 256, 0, ctx->stream>>>(a);
            s = post_launch(ctx, "ply_decode_compressed_kernel");
        }
    }
    release_all();
    return s;
}

// Header of splat_to_ply (export.rs:170-191) with the rows' byte count.
static std::string export_header(uint32_t n, uint32_t coeffs, int32_t mip, const float* up_axis) {
    auto fmt = [](float v) {
        char buf[32];
        auto r = std::to_chars(buf, buf + sizeof buf, v);
        return std::string(buf, r.ptr);
    };
    std::string h = "ply\nformat binary_little_endian 1.0\ncomment Exported from Brush\n";
    if (up_axis) h += "comment Vertical axis: " + fmt(up_axis[0]) + " " + fmt(up_axis[1]) + " " + fmt(up_axis[2]) + "\n";
    else h += "comment Vertical axis: y\n";
    uint32_t degree = 0;
    while ((degree + 1) * (degree + 1) < coeffs) ++degree;
    h += "comment SH degree: " + std::to_string(degree) + "\n";
    h += std::string("comment SplatRenderMode: ") + (mip ? "mip" : "default") + "\n";
    h += "element vertex " + std::to_string(n) + "\n";
    static const char* names[14] = {"x", "y", "z", "scale_0", "scale_1", "scale_2", "opacity",
                                    "rot_0", "rot_1", "rot_2", "rot_3", "f_dc_0", "f_dc_1", "f_dc_2"};
    for (const char* nm : names) h += std::string("property float ") + nm + "\n";
    for (uint32_t k = 0; k < 3 * (coeffs - 1); ++k) h += "property float f_rest_" + std::to_string(k) + "\n";
    h += "end_header\n";
    return h;
}

bsx_status bsx_ply_export_size(uint32_t n, uint32_t coeffs, int32_t mip, const float* up_axis, uint64_t* bytes) {
    if (!bytes || !(coeffs == 1 || coeffs == 4 || coeffs == 9 || coeffs == 16)) return BSX_ERR_INVALID_ARG;
    *bytes = export_header(n, coeffs, mip, up_axis).size() + (uint64_t)n * (14 + 3 * (coeffs - 1)) * 4;
    return BSX_OK;
}

bsx_status bsx_ply_export(bsx_ctx* ctx, const float* d_transforms, const float* d_sh, const float* d_raw_opac,
                          uint32_t n, uint32_t coeffs, int32_t mip, const float* up_axis, uint8_t* host_out,
                          uint64_t capacity, uint64_t* written) {
    using namespace bsx;
    if (!ctx || !host_out || !written || (n && (!d_transforms || !d_sh || !d_raw_opac))) return BSX_ERR_INVALID_ARG;
    if (!(coeffs == 1 || coeffs == 4 || coeffs == 9 || coeffs == 16))
        return fail(ctx, BSX_ERR_INVALID_ARG, "export supports SH degrees 0-3");
    cudaSetDevice(ctx->device);
    const std::string h = export_header(n, coeffs, mip, up_axis);
    const uint64_t rows = (uint64_t)n * (14 + 3 * (coeffs - 1)) * 4;
    if (h.size() + rows > capacity) return fail(ctx, BSX_ERR_CAPACITY, "export buffer too small");
    std::memcpy(host_out, h.data(), h.size());
    *written = h.size() + rows;
    if (!n) return BSX_OK;
    uint8_t* d_rows = nullptr;
    bsx_status s = check_cuda(ctx, cudaMallocAsync((void**)&d_rows, rows, ctx->stream), "ply export staging");
    if (s != BSX_OK) return s;
    EncArgs a{d_transforms, d_sh, d_raw_opac, n, coeffs, d_rows};
    prof_begin(ctx);
    ply_encode_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(a);
    s = post_launch(ctx, "ply_encode_kernel");
    if (s == BSX_OK)
        s = check_cuda(ctx, cudaMemcpyAsync(host_out + h.size(), d_rows, rows, cudaMemcpyDeviceToHost, ctx->stream),
                       "ply export read-back");
    cudaFreeAsync(d_rows, ctx->stream);
    if (s == BSX_OK) s = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "ply export sync");
    return s;
}

}  // extern "C"
