// refine.cpp - CPU restatement of the reference's densification step.
//
// TEST INFRASTRUCTURE ONLY (see oracle.cpp). Restates, on the host and one
// splat at a time, SplatTrainer::refine_for_phase / refine_splats /
// prune_points (crates/brush-train/src/train.rs:1191-1860) with the growth
// signal taken from the gradient norm. Each per-element expression follows
// the reference's tensor expression in the same operation order, so the CUDA
// implementation (brush_b200/csrc/refine.cu), written separately in the same
// order, must agree bit for bit.
//
// Sampling: the reference calls rand::seq::index::sample_weighted (weighted
// sampling without replacement, multinomial.rs:1-33) on rand's StdRng. This
// restatement uses the same algorithm family (Efraimidis-Spirakis keys: the k
// largest of log(u_i) / w_i) with a counter-based generator, u_i from
// SplitMix64(seed, refine count, stream, i); ties go to the lower index.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <set>
#include <vector>

#include "../include/bsx.h"
#include "../include/bsx_fmath.h"

namespace {

uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform in (0, 1] with 24 random bits.
float uniform01(uint64_t seed, uint32_t stream, uint32_t index) {
    const uint64_t h = splitmix64(seed ^ splitmix64(((uint64_t)stream << 32) | index));
    return (float)((h >> 40) + 1) * 5.9604644775390625e-08f;  // 2^-24
}

// k largest keys log(u)/w among positive finite weights (lower index first on ties).
std::vector<uint32_t> weighted_sample(const std::vector<float>& w, uint32_t k, uint64_t seed, uint32_t stream) {
    std::vector<std::pair<float, uint32_t>> keys;
    for (uint32_t i = 0; i < (uint32_t)w.size(); ++i) {
        const float wi = w[i];
        if (!(wi > 0.0f) || !bsx_is_finite(wi)) continue;
        keys.push_back({bsx_logf(uniform01(seed, stream, i)) / wi, i});
    }
    std::stable_sort(keys.begin(), keys.end(), [](const auto& a, const auto& b) { return a.first > b.first; });
    std::vector<uint32_t> out;
    for (uint32_t j = 0; j < k && j < keys.size(); ++j) out.push_back(keys[j].second);
    return out;
}

float sigmoid(float x) { return bsx_sigmoid(x); }
float inv_sigmoid(float x) { return bsx_logf(x / (1.0f - x)); }  // train.rs:137-139
float clampf(float x, float lo, float hi) { return bsx_min(bsx_max(x, lo), hi); }
uint32_t sat_sub(uint32_t a, uint32_t b) { return a > b ? a - b : 0u; }

struct Plan {
    uint32_t n = 0, coeffs = 0, refine_count = 0;
    std::vector<uint32_t> keep;   // kept original indices, ascending
    std::vector<uint32_t> split;  // split rows in the kept numbering, ascending
    std::vector<uint32_t> clone;  // gradient-threshold rule: cloned rows (kept numbering), ascending
    std::vector<float> screen;    // max_screen_size of the kept rows
    bsx_refine_config cfg{};
    bsx_refine_stats stats{};
};

// The gradient-threshold rule (the original 3D Gaussian splatting trainer's
// densify_and_clone / densify_and_split, Kerbl et al. 2023) on the kept rows:
// average view-space gradient norm = accum / visible steps (0 where never
// visible) >= threshold selects a row; a selected row whose largest scale is
// at most percent_dense x the largest bounds extent is cloned, any other is
// split; clones then splits are cut to the max_splats budget in row order.
void plan_grad_threshold(Plan* p, const float* t, const float* vis, const float* grad2d, float max_extent) {
    const bsx_refine_config& c = p->cfg;
    const uint32_t K = (uint32_t)p->keep.size();
    const float dense = c.percent_dense * max_extent;
    std::vector<uint32_t> clone, split;
    for (uint32_t j = 0; j < K; ++j) {
        const uint32_t i = p->keep[j];
        const float avg = vis[i] > 0.0f ? grad2d[i] / vis[i] : 0.0f;
        if (!(avg >= c.growth_grad_threshold)) continue;
        const float* r = t + (size_t)i * 10;
        const float smax = bsx_max(bsx_max(bsx_expf(r[7]), bsx_expf(r[8])), bsx_expf(r[9]));
        (smax <= dense ? clone : split).push_back(j);
    }
    uint32_t budget = sat_sub(c.max_splats, K);
    if (clone.size() > budget) clone.resize(budget);
    budget -= (uint32_t)clone.size();
    if (split.size() > budget) split.resize(budget);
    p->clone = clone;
    p->split = split;
}

// Rows of the gradient-threshold rule: kept rows that are not split (in order),
// clones, first children, second children. Split children: mean + R(q) (s * n)
// with n = bsx_normal3(seed, stream, kept row), stream 2^30 + 2 refine_count + k
// for child k, R the rotation of the normalised quaternion, s = exp(log-scale);
// log-scale log(s / 1.6); rotation, SH and opacity copied. New rows have zero
// moments.
void apply_grad_threshold(const Plan* p, const float* t, const float* sh, const float* op, const float* m_t,
                          const float* m_s, const float* m_o, const float* v_t, const float* v_s, const float* v_o,
                          float* nt, float* nsh, float* nop, float* nm_t, float* nm_s, float* nm_o, float* nv_t,
                          float* nv_s, float* nv_o) {
    const uint32_t K = (uint32_t)p->keep.size(), C = (uint32_t)p->clone.size(), S = (uint32_t)p->split.size();
    const uint32_t c3 = 3 * p->coeffs;
    std::vector<uint8_t> is_split(K, 0);
    for (uint32_t j : p->split) is_split[j] = 1;
    auto zero_moments = [&](uint32_t r) {
        memset(nm_t + (size_t)r * 10, 0, 40);
        memset(nm_s + (size_t)r * c3, 0, (size_t)c3 * 4);
        nm_o[r] = 0.0f;
        memset(nv_t + (size_t)r * 10, 0, 40);
        nv_s[r] = 0.0f;
        nv_o[r] = 0.0f;
    };
    uint32_t r = 0;
    for (uint32_t j = 0; j < K; ++j) {
        if (is_split[j]) continue;
        const uint32_t i = p->keep[j];
        memcpy(nt + (size_t)r * 10, t + (size_t)i * 10, 40);
        memcpy(nsh + (size_t)r * c3, sh + (size_t)i * c3, (size_t)c3 * 4);
        nop[r] = op[i];
        memcpy(nm_t + (size_t)r * 10, m_t + (size_t)i * 10, 40);
        memcpy(nm_s + (size_t)r * c3, m_s + (size_t)i * c3, (size_t)c3 * 4);
        nm_o[r] = m_o[i];
        memcpy(nv_t + (size_t)r * 10, v_t + (size_t)i * 10, 40);
        nv_s[r] = v_s[i];
        nv_o[r] = v_o[i];
        ++r;
    }
    for (uint32_t q = 0; q < C; ++q, ++r) {
        const uint32_t i = p->keep[p->clone[q]];
        memcpy(nt + (size_t)r * 10, t + (size_t)i * 10, 40);
        memcpy(nsh + (size_t)r * c3, sh + (size_t)i * c3, (size_t)c3 * 4);
        nop[r] = op[i];
        zero_moments(r);
    }
    for (uint32_t k = 0; k < 2; ++k)
        for (uint32_t q = 0; q < S; ++q, ++r) {
            const uint32_t j = p->split[q], i = p->keep[j];
            const float* pr = t + (size_t)i * 10;
            const float mag = bsx_max(sqrtf(pr[3] * pr[3] + pr[4] * pr[4] + pr[5] * pr[5] + pr[6] * pr[6]), 1e-32f);
            const float qw = pr[3] / mag, qx = pr[4] / mag, qy = pr[5] / mag, qz = pr[6] / mag;
            float z[3];
            bsx_normal3(p->cfg.seed, (1u << 30) + 2 * p->refine_count + k, j, z);
            const float vx = bsx_expf(pr[7]) * z[0], vy = bsx_expf(pr[8]) * z[1], vz = bsx_expf(pr[9]) * z[2];
            const float qw2 = qw * qw, qx2 = qx * qx, qy2 = qy * qy, qz2 = qz * qz;
            const float xy = qx * qy, xz = qx * qz, yz = qy * qz, wx = qw * qx, wy = qw * qy, wz = qw * qz;
            const float d[3] = {
                (qw2 + qx2 - qy2 - qz2) * vx + (xy * vy + xz * vz + wy * vz - wz * vy) * 2.0f,
                (qw2 - qx2 + qy2 - qz2) * vy + (xy * vx + yz * vz + wz * vx - wx * vz) * 2.0f,
                (qw2 - qx2 - qy2 + qz2) * vz + (xz * vx + yz * vy + wx * vy - wy * vx) * 2.0f};
            float* cr = nt + (size_t)r * 10;
            for (int a = 0; a < 3; ++a) cr[a] = pr[a] + d[a];
            for (int a = 0; a < 4; ++a) cr[3 + a] = pr[3 + a];
            for (int a = 0; a < 3; ++a) cr[7 + a] = bsx_logf(bsx_expf(pr[7 + a]) / 1.6f);
            memcpy(nsh + (size_t)r * c3, sh + (size_t)i * c3, (size_t)c3 * 4);
            nop[r] = op[i];
            zero_moments(r);
        }
}

}  // namespace

extern "C" {

// Prune decision bits per splat (train.rs:1258-1350): 1 alpha < min_opacity,
// 2 a scale > max_allowed, 4 outside the bounds, 8 a non-finite parameter,
// 16 a raw scale < min_scale_prune_threshold, 32 |q|^2 < 1e-8.
void orc_refine_prune_mask(const float* t, const float* sh, const float* op, uint32_t n, uint32_t coeffs,
                           const bsx_refine_config* cfg, const float center[3], float max_allowed, uint8_t* out) {
    const uint32_t c3 = 3 * coeffs;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        const float* r = t + i * 10;
        uint8_t m = 0;
        if (sigmoid(op[i]) < cfg->min_opacity) m |= 1;
        bool big = false;
        for (int k = 0; k < 3; ++k) big |= bsx_expf(r[7 + k]) > max_allowed;
        if (big) m |= 2;
        bool out_b = false;
        if (cfg->radial_bounds_prune) {
            const float dx = r[0] - center[0], dy = r[1] - center[1], dz = r[2] - center[2];
            out_b = sqrtf(dx * dx + dy * dy + dz * dz) > max_allowed;
        } else {
            for (int k = 0; k < 3; ++k) out_b |= fabsf(r[k] - center[k]) > max_allowed;
        }
        if (out_b) m |= 4;
        bool bad = !bsx_is_finite(op[i]);
        for (int k = 0; k < 10; ++k) bad |= !bsx_is_finite(r[k]);
        for (uint32_t k = 0; k < c3; ++k) bad |= !bsx_is_finite(sh[i * c3 + k]);
        if (bad) m |= 8;
        if (cfg->min_scale_prune) {
            bool small = false;
            for (int k = 0; k < 3; ++k) small |= bsx_expf(r[7 + k]) < cfg->min_scale_prune_threshold;
            if (small) m |= 16;
        }
        if (cfg->near_zero_rotation_prune) {
            const float qn = r[3] * r[3] + r[4] * r[4] + r[5] * r[5] + r[6] * r[6];
            if (qn < 1e-8f) m |= 32;
        }
        out[i] = m;
    }
}

// Decide the refine (train.rs:1258-1500). refine_norm / vis / screen are the
// RefineRecord arrays. Returns a plan handle; stats filled.
void* orc_refine_plan2(const float* t, const float* sh, const float* op, const float* refine_norm, const float* vis,
                       const float* screen, const float* grad2d, uint32_t n, uint32_t coeffs,
                       const bsx_refine_config* cfg, const float center[3], const float extent[3],
                       uint32_t global_iter, uint32_t refine_count, bsx_refine_stats* stats) {
    Plan* p = new Plan();
    p->n = n;
    p->coeffs = coeffs;
    p->cfg = *cfg;
    p->refine_count = refine_count;
    const float max_extent = bsx_max(bsx_max(extent[0], extent[1]), extent[2]);
    const float max_allowed = max_extent * cfg->prune_extent_factor;
    std::vector<uint8_t> mask(n);
    orc_refine_prune_mask(t, sh, op, n, coeffs, cfg, center, max_allowed, mask.data());
    uint32_t non_finite = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (mask[i] & 8) ++non_finite;
        if (!mask[i]) p->keep.push_back(i);
    }
    // prune_points keeps every splat when all would go (train.rs:1830-1833)
    const bool all_pruned = p->keep.empty() && n > 0;
    if (all_pruned)
        for (uint32_t i = 0; i < n; ++i) p->keep.push_back(i);
    const uint32_t K = (uint32_t)p->keep.size();
    const uint32_t pruned = n - K;
    if (cfg->rule == BSX_REFINE_GRAD_THRESHOLD) {
        plan_grad_threshold(p, t, vis, grad2d, max_extent);
        bsx_refine_stats& st = p->stats;
        const uint32_t C = (uint32_t)p->clone.size(), S = (uint32_t)p->split.size();
        st.num_added = C + S;
        st.num_split_oversized = 0;
        st.num_split_high_grad = S;
        st.num_pruned = all_pruned ? 0 : pruned;
        st.num_pruned_non_finite = non_finite;
        st.total_splats = K + C + S;
        if (stats) *stats = st;
        return p;
    }
    std::vector<float> vis_k(K), rn_k(K), op_k(K);
    p->screen.resize(K);
    for (uint32_t j = 0; j < K; ++j) {
        const uint32_t i = p->keep[j];
        vis_k[j] = vis[i];
        rn_k[j] = refine_norm[i];
        op_k[j] = op[i];
        p->screen[j] = screen[i];
    }
    std::set<uint32_t> split;
    const uint64_t seed = cfg->seed;
    if (pruned > 0) {  // replacement weighted by opacity x visibility (train.rs:1368-1392)
        std::vector<float> w(K);
        for (uint32_t j = 0; j < K; ++j) w[j] = sigmoid(op_k[j]) * (vis_k[j] > 0.0f ? 1.0f : 0.0f);
        for (uint32_t s : weighted_sample(w, pruned, seed, 2 * refine_count)) split.insert(s);
    }
    const uint32_t pre_oversized = (uint32_t)split.size();
    if (cfg->split_at_screen_size > 0.0f) {  // train.rs:1398-1424
        uint32_t budget = sat_sub(cfg->max_splats, K + (uint32_t)split.size());
        for (uint32_t j = 0; j < K && budget > 0; ++j)
            if (p->screen[j] > cfg->split_at_screen_size && vis_k[j] > 0.0f)
                if (split.insert(j).second) --budget;
    }
    const uint32_t num_oversized = (uint32_t)split.size() - pre_oversized;
    const uint32_t pre_grow = (uint32_t)split.size();
    if (global_iter < cfg->growth_stop_iter) {  // train.rs:1428-1495, gradient signal
        std::vector<float> w(K);
        uint32_t count = 0;
        for (uint32_t j = 0; j < K; ++j) {
            const bool above = rn_k[j] > cfg->growth_grad_threshold && vis_k[j] > 0.0f;
            count += above;
            w[j] = (above ? 1.0f : 0.0f) * rn_k[j];
        }
        const uint32_t grow_count = (uint32_t)roundf((float)count * cfg->growth_select_fraction);
        const uint32_t sample_high = sat_sub(grow_count, pruned);
        const uint32_t headroom = sat_sub(cfg->max_splats, K + (uint32_t)split.size());
        const uint32_t grow = std::min(sample_high, headroom);
        if (grow > 0)
            for (uint32_t s : weighted_sample(w, grow, seed, 2 * refine_count + 1)) split.insert(s);
    }
    p->split.assign(split.begin(), split.end());
    bsx_refine_stats& st = p->stats;
    st.num_added = (uint32_t)p->split.size();
    st.num_split_oversized = num_oversized;
    st.num_split_high_grad = (uint32_t)split.size() - pre_grow;
    st.num_pruned = all_pruned ? 0 : pruned;
    st.num_pruned_non_finite = non_finite;
    st.total_splats = K + (uint32_t)p->split.size();
    if (stats) *stats = st;
    return p;
}

void* orc_refine_plan(const float* t, const float* sh, const float* op, const float* refine_norm, const float* vis,
                      const float* screen, uint32_t n, uint32_t coeffs, const bsx_refine_config* cfg,
                      const float center[3], const float extent[3], uint32_t global_iter, uint32_t refine_count,
                      bsx_refine_stats* stats) {
    return orc_refine_plan2(t, sh, op, refine_norm, vis, screen, nullptr, n, coeffs, cfg, center, extent, global_iter,
                            refine_count, stats);
}

// Kept and split rows (kept numbering) of a plan.
void orc_refine_plan_rows(void* h, uint32_t* keep_out, uint32_t* split_out) {
    const Plan* p = (const Plan*)h;
    memcpy(keep_out, p->keep.data(), p->keep.size() * 4);
    memcpy(split_out, p->split.data(), p->split.size() * 4);
}

// Apply a plan (train.rs:1536-1740 and prune_points :1811-1860). Moments: m_t
// [n,10], m_s [n,3C], m_o [n]; v_t [n,10], v_s [n], v_o [n]; the outputs have
// the new count.
void orc_refine_apply(void* h, const float* t, const float* sh, const float* op, const float* m_t, const float* m_s,
                      const float* m_o, const float* v_t, const float* v_s, const float* v_o, float* nt, float* nsh,
                      float* nop, float* nm_t, float* nm_s, float* nm_o, float* nv_t, float* nv_s, float* nv_o,
                      uint32_t phase_iter, uint32_t phase_total) {
    const Plan* p = (const Plan*)h;
    const bsx_refine_config& c = p->cfg;
    if (c.rule == BSX_REFINE_GRAD_THRESHOLD) {
        apply_grad_threshold(p, t, sh, op, m_t, m_s, m_o, v_t, v_s, v_o, nt, nsh, nop, nm_t, nm_s, nm_o, nv_t, nv_s,
                             nv_o);
        return;
    }
    const uint32_t K = (uint32_t)p->keep.size(), S = (uint32_t)p->split.size(), c3 = 3 * p->coeffs;
    // prune_points: select kept rows of the splats and of both moments
    for (uint32_t j = 0; j < K; ++j) {
        const uint32_t i = p->keep[j];
        memcpy(nt + (size_t)j * 10, t + (size_t)i * 10, 40);
        memcpy(nsh + (size_t)j * c3, sh + (size_t)i * c3, (size_t)c3 * 4);
        nop[j] = op[i];
        memcpy(nm_t + (size_t)j * 10, m_t + (size_t)i * 10, 40);
        memcpy(nm_s + (size_t)j * c3, m_s + (size_t)i * c3, (size_t)c3 * 4);
        nm_o[j] = m_o[i];
        memcpy(nv_t + (size_t)j * 10, v_t + (size_t)i * 10, 40);
        nv_s[j] = v_s[i];
        nv_o[j] = v_o[i];
    }
    const float ln_other = bsx_logf(c.split_other_axis_scale);
    for (uint32_t q = 0; q < S; ++q) {
        const uint32_t s = p->split[q], child = K + q;
        float* pr = nt + (size_t)s * 10;
        const float mean[3] = {pr[0], pr[1], pr[2]};
        const float qr[4] = {pr[3], pr[4], pr[5], pr[6]};
        const float ls[3] = {pr[7], pr[8], pr[9]};
        const float raw_op = nop[s];
        // train.rs:1562-1567: normalised rotation
        const float mag = bsx_max(sqrtf(qr[0] * qr[0] + qr[1] * qr[1] + qr[2] * qr[2] + qr[3] * qr[3]), 1e-32f);
        const float rot[4] = {qr[0] / mag, qr[1] / mag, qr[2] / mag, qr[3] / mag};
        const float sc[3] = {bsx_expf(ls[0]), bsx_expf(ls[1]), bsx_expf(ls[2])};
        // :1586-1589 opacity of both halves
        const float new_opac = sigmoid(raw_op) * c.split_opacity_scale;
        const float new_raw = inv_sigmoid(clampf(new_opac, c.min_opacity, 1.0f - c.min_opacity));
        // :1594-1602 longest log-scale axis (first maximum)
        int L = 0;
        for (int k = 1; k < 3; ++k)
            if (ls[k] > ls[L]) L = k;
        // :1610-1621 longest-axis shrink
        float m_long = c.split_long_axis_scale;
        if (c.split_at_screen_size > 0.0f)
            m_long = bsx_min((1.0f / bsx_max(p->screen[s], 1e-6f)) * c.split_at_screen_size, c.split_long_axis_scale);
        // :1629-1630 offset = rotate(q, e_L * scale_L * split_long_axis_scale)
        float off[3];
        for (int k = 0; k < 3; ++k) off[k] = ((k == L ? 1.0f : 0.0f) * sc[k]) * c.split_long_axis_scale;
        const float qw = rot[0], qx = rot[1], qy = rot[2], qz = rot[3];
        const float vx = off[0], vy = off[1], vz = off[2];
        // quat_vec.rs:4-44
        const float qw2 = qw * qw, qx2 = qx * qx, qy2 = qy * qy, qz2 = qz * qz;
        const float xy = qx * qy, xz = qx * qz, yz = qy * qz, wx = qw * qx, wy = qw * qy, wz = qw * qz;
        const float smp[3] = {
            (qw2 + qx2 - qy2 - qz2) * vx + (xy * vy + xz * vz + wy * vz - wz * vy) * 2.0f,
            (qw2 - qx2 + qy2 - qz2) * vy + (xy * vx + yz * vz + wz * vx - wx * vz) * 2.0f,
            (qw2 - qx2 - qy2 + qz2) * vz + (xz * vx + yz * vy + wx * vy - wy * vx) * 2.0f};
        // :1637-1645 new log-scales
        const float ln_long = bsx_logf(m_long);
        float nls[3];
        for (int k = 0; k < 3; ++k) {
            const float oh = k == L ? 1.0f : 0.0f;
            const float base = ls[k] + ln_other, lng = ls[k] + ln_long;
            nls[k] = base * (-oh + 1.0f) + lng * oh;
        }
        // :1651-1664 parent: scatter-add of the differences
        for (int k = 0; k < 3; ++k) {
            pr[k] = mean[k] + (-smp[k]);
            pr[7 + k] = ls[k] + (nls[k] - ls[k]);
        }
        for (int k = 0; k < 4; ++k) pr[3 + k] = qr[k] + 0.0f;
        nop[s] = raw_op + (new_raw - raw_op);
        // :1669-1670 child row
        float* cr = nt + (size_t)child * 10;
        for (int k = 0; k < 3; ++k) cr[k] = mean[k] + smp[k];
        for (int k = 0; k < 4; ++k) cr[3 + k] = rot[k];
        for (int k = 0; k < 3; ++k) cr[7 + k] = nls[k];
        memcpy(nsh + (size_t)child * c3, nsh + (size_t)s * c3, (size_t)c3 * 4);
        nop[child] = new_raw;
        // :1684-1725 both halves start with zero moments (parent: x + (-x))
        for (int k = 0; k < 10; ++k) {
            nm_t[(size_t)s * 10 + k] = nm_t[(size_t)s * 10 + k] + (-nm_t[(size_t)s * 10 + k]);
            nv_t[(size_t)s * 10 + k] = nv_t[(size_t)s * 10 + k] + (-nv_t[(size_t)s * 10 + k]);
            nm_t[(size_t)child * 10 + k] = 0.0f;
            nv_t[(size_t)child * 10 + k] = 0.0f;
        }
        for (uint32_t k = 0; k < c3; ++k) {
            nm_s[(size_t)s * c3 + k] = nm_s[(size_t)s * c3 + k] + (-nm_s[(size_t)s * c3 + k]);
            nm_s[(size_t)child * c3 + k] = 0.0f;
        }
        nv_s[s] = nv_s[s] + (-nv_s[s]);
        nv_s[child] = 0.0f;
        nm_o[s] = nm_o[s] + (-nm_o[s]);
        nv_o[s] = nv_o[s] + (-nv_o[s]);
        nm_o[child] = 0.0f;
        nv_o[child] = 0.0f;
    }
    // :1702-1740 opacity and scale decay over every row
    const float train_t = clampf((float)phase_iter / (float)std::max(phase_total, 1u), 0.0f, 1.0f);
    const float t_shrink = 1.0f - train_t;
    const float minus_opac = c.opac_decay * t_shrink;
    const float scale_factor = 1.0f - c.scale_decay * t_shrink;
    for (uint32_t r = 0; r < K + S; ++r) {
        const float new_op = sigmoid(nop[r]) - minus_opac;
        nop[r] = inv_sigmoid(clampf(new_op, 1e-12f, 1.0f - 1e-12f));
        if (c.scale_decay > 0.0f)
            for (int k = 0; k < 3; ++k) {
                float* v = nt + (size_t)r * 10 + 7 + k;
                *v = bsx_logf(bsx_max(bsx_expf(*v) * scale_factor, 1e-12f));
            }
    }
}

void orc_refine_free(void* h) { delete (Plan*)h; }

float orc_refine_uniform(uint64_t seed, uint32_t stream, uint32_t index) { return uniform01(seed, stream, index); }

// The weighted sampler alone: up to k distinct indices, in key order. Returns the count.
uint32_t orc_weighted_sample(const float* w, uint32_t n, uint32_t k, uint64_t seed, uint32_t stream, uint32_t* out) {
    const std::vector<uint32_t> r = weighted_sample(std::vector<float>(w, w + n), k, seed, stream);
    std::copy(r.begin(), r.end(), out);
    return (uint32_t)r.size();
}

}  // extern "C"
