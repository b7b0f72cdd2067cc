// trainer.cuh - the native trainer's state (internal; shared by train.cu and refine.cu).
#pragma once
#include "common.cuh"

struct bsx_trainer {
    bsx_ctx* ctx = nullptr;
    uint32_t n = 0, coeffs = 0;
    bsx_train_config cfg{};
    bsx::DevBuf grads, v_combined, v_output, stats, moments;
    uint32_t moment_rows = 0;  // rows the moments cover (all, or this rank's shard)
    int moment_world = 0, moment_rank = -1;
    uint32_t step = 0;
    double mean_prev = 0.0, mean_gamma = 1.0, scale_prev = 0.0, scale_gamma = 1.0;
    uint32_t dp_epoch = 0;
    int keep_grads = 0;  // bsx_train_step also writes the dense gradients
    // densification: the plan of the last bsx_trainer_refine_plan
    bool planned = false;
    uint32_t plan_n = 0, plan_kept = 0, plan_split_count = 0, plan_clone_count = 0, refines = 0;
    bsx_refine_config plan_cfg{};
    bsx::DevBuf plan_keep, plan_split, plan_scratch, moments_next;
};

namespace bsx {

// RefineRecord arrays per splat: refine-weight MAX, visibility SUM, screen-size
// MAX, view-space gradient-norm SUM (the gradient-threshold densification rule).
constexpr size_t kRecordArrays = 4;

// Moment views over one buffer of `rows` rows:
// m: [rows,10] | [rows,3C] | [rows,1]; v: [rows,10] | [rows] | [rows,1],
// each array starting on a 16-byte boundary (vector loads in the updates).
inline size_t round4(size_t x) { return (x + 3) / 4 * 4; }
inline void moment_views(float* base, uint32_t rows, uint32_t coeffs, float** m, float** v) {
    const size_t c3 = 3 * (size_t)coeffs;
    m[0] = base;
    m[1] = m[0] + round4((size_t)rows * 10);
    m[2] = m[1] + round4((size_t)rows * c3);
    v[0] = m[2] + round4(rows);
    v[1] = v[0] + round4((size_t)rows * 10);
    v[2] = v[1] + round4(rows);
}

inline size_t moment_floats(uint32_t rows, uint32_t coeffs) {
    const size_t c3 = 3 * (size_t)coeffs;
    return round4((size_t)rows * 10) + round4((size_t)rows * c3) + round4(rows) + round4((size_t)rows * 10) +
           round4(rows) + round4(rows);
}

}  // namespace bsx
