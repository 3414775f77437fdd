// model.cpp — host-side model logic of the training step: camera setup
// (Model::prepareCam, core/src/model.cpp:500-544) and the learning-rate
// schedule (Model::schedulersStep, core/src/model.cpp:183-186).
//
// Compiled with -ffp-contract=off so the matrices are the same floats the
// reference's C++ computes (plain IEEE multiply/add in source order).
#include <algorithm>
#include <cmath>
#include <cstring>

#include "msplat_backend.h"

extern "C" {

int msplat_prepare_camera(const float camToWorld[16], float fx, float fy, float cx, float cy, int32_t width,
                          int32_t height, MsplatCamera* out) {
    if (!camToWorld || !out || width <= 0 || height <= 0 || !(fx > 0.f) || !(fy > 0.f)) return MSPLAT_ERR_ARGUMENT;
    const float fovX = 2.0f * std::atan(width / (2.0f * fx));
    const float fovY = 2.0f * std::atan(height / (2.0f * fy));
    const float* d = camToWorld;
    // OpenGL -> OpenCV camera: flip the y and z columns of the rotation.
    float R[3][3], Rinv[3][3], T[3], Tinv[3];
    for (int i = 0; i < 3; i++) {
        R[i][0] = d[i * 4 + 0];
        R[i][1] = -d[i * 4 + 1];
        R[i][2] = -d[i * 4 + 2];
        T[i] = d[i * 4 + 3];
    }
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) Rinv[i][j] = R[j][i];
    for (int i = 0; i < 3; i++) Tinv[i] = -(Rinv[i][0] * T[0] + Rinv[i][1] * T[1] + Rinv[i][2] * T[2]);
    const float vm[16] = {Rinv[0][0], Rinv[0][1], Rinv[0][2], Tinv[0], Rinv[1][0], Rinv[1][1], Rinv[1][2], Tinv[1],
                          Rinv[2][0], Rinv[2][1], Rinv[2][2], Tinv[2], 0, 0, 0, 1};
    // Perspective with znear 0.001, zfar 1000.
    const float t_p = 0.001f * std::tan(0.5f * fovY), r_p = 0.001f * std::tan(0.5f * fovX);
    const float pm[16] = {0.001f / r_p, 0, 0, 0, 0, 0.001f / t_p, 0, 0, 0, 0,
                          (1000.0f + 0.001f) / (1000.0f - 0.001f), -1000.0f * 0.001f / (1000.0f - 0.001f),
                          0, 0, 1, 0};
    float pvm[16] = {};
    for (int i = 0; i < 4; i++)
        for (int j = 0; j < 4; j++)
            for (int k = 0; k < 4; k++) pvm[i * 4 + j] += pm[i * 4 + k] * vm[k * 4 + j];
    std::memcpy(out->viewmat, vm, sizeof(vm));
    std::memcpy(out->projmat, pvm, sizeof(pvm));
    out->fx = fx;
    out->fy = fy;
    out->cx = cx;
    out->cy = cy;
    out->width = width;
    out->height = height;
    out->cam_pos[0] = T[0];
    out->cam_pos[1] = T[1];
    out->cam_pos[2] = T[2];
    return MSPLAT_OK;
}

float msplat_means_lr(int32_t step, int32_t max_steps, float lr_init, float lr_final) {
    // Log-linear decay of the means learning rate.
    const float t = std::clamp((float)step / (float)max_steps, 0.f, 1.f);
    return std::exp(std::log(lr_init) * (1.f - t) + std::log(lr_final) * t);
}

}  // extern "C"
