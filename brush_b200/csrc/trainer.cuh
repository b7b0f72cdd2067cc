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
    // densification: the plan of the last bsx_trainer_refine_plan
    bool planned = false;
    uint32_t plan_n = 0, plan_kept = 0, plan_split_count = 0, refines = 0;
    bsx_refine_config plan_cfg{};
    bsx::DevBuf plan_keep, plan_split, plan_scratch, moments_next;
};

namespace bsx {

// Moment views over one buffer of `rows` rows:
// m: [rows,10] | [rows,3C] | [rows,1]; v: [rows,10] | [rows] | [rows,1].
inline void moment_views(float* base, uint32_t rows, uint32_t coeffs, float** m, float** v) {
    const size_t c3 = 3 * (size_t)coeffs;
    m[0] = base;
    m[1] = m[0] + (size_t)rows * 10;
    m[2] = m[1] + (size_t)rows * c3;
    v[0] = m[2] + rows;
    v[1] = v[0] + (size_t)rows * 10;
    v[2] = v[1] + rows;
}

inline size_t moment_floats(uint32_t rows, uint32_t coeffs) {
    return (size_t)rows * (10 + 3 * (size_t)coeffs + 1) + (size_t)rows * (10 + 1 + 1);
}

}  // namespace bsx
