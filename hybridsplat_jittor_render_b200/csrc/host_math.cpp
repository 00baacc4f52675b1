// Host-side FP32 math that must round exactly like the reference's host code.
//
// The reference computes these on x86-64 with g++ and no FMA instructions
// (baseline ISA), so every product and sum is an individually rounded IEEE
// single operation in source order. This file is compiled with
// -ffp-contract=off and no -march flag to keep that property.
//
//  - flashgs_camera_matrices: getViewMatrix / getProjectionMatrix and the
//    GLM mat4 product (vendor/flashgs/cuda_rasterizer/preprocess.cu:599-627,
//    glm/detail/type_mat4x4.inl:630-649).
//  - flashgs_prepare_host: hs_flashgs_prepare_npz_host_f32_v1
//    (rasterizer/flashgs_prepare.cpp:30-84, vendor/flashgs/model_utils.h:10-43)
//    with glm::normalize as v * (1 / sqrt(dot(v, v))) and the vec4 dot as
//    (x*x + y*y) + (z*z + w*w) (glm/detail/func_geometric.inl:58-90).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "context.h"

namespace hs {

void flashgs_camera_matrices(const float position[3], const float rotation9[9], int width,
                             int height, float focal_x, float focal_y, float z_far,
                             float z_near, float view[16], float proj[16]) {
    // rotation9 rows become glm::mat3 columns: rot[c][i] = rotation9[3c + i]
    // (flashgs_backend.cu:426-430).
    std::memset(view, 0, 16 * sizeof(float));
    for (int c = 0; c < 3; ++c) {
        for (int i = 0; i < 3; ++i) view[4 * c + i] = rotation9[3 * c + i];
    }
    const float nx = -position[0], ny = -position[1], nz = -position[2];
    for (int i = 0; i < 3; ++i) {
        float t = rotation9[i] * nx;
        t = t + rotation9[3 + i] * ny;
        t = t + rotation9[6 + i] * nz;
        view[12 + i] = t;
    }
    view[15] = 1.0f;

    const float top = static_cast<float>(height) / (2.0f * focal_y) * z_near;
    const float bottom = -top;
    const float right = static_cast<float>(width) / (2.0f * focal_x) * z_near;
    const float left = -right;
    float p[16];  // GLM P[c][r] at p[4c + r]
    std::memset(p, 0, sizeof(p));
    const float z_sign = 1.0f;
    p[0 * 4 + 0] = 2.0f * z_near / (right - left);
    p[1 * 4 + 1] = 2.0f * z_near / (top - bottom);
    p[0 * 4 + 2] = (right + left) / (right - left);
    p[1 * 4 + 2] = (top + bottom) / (top - bottom);
    p[3 * 4 + 2] = z_sign;
    p[2 * 4 + 2] = z_sign * z_far / (z_far - z_near);
    p[2 * 4 + 3] = -(z_far * z_near) / (z_far - z_near);
    // A = transpose(P): A[c][r] = P[r][c]; result[j] = A0*V[j][0] + A1*V[j][1] + A2*V[j][2] + A3*V[j][3]
    float a[16];
    for (int c = 0; c < 4; ++c) {
        for (int r = 0; r < 4; ++r) a[4 * c + r] = p[4 * r + c];
    }
    for (int j = 0; j < 4; ++j) {
        for (int r = 0; r < 4; ++r) {
            float t = a[0 * 4 + r] * view[4 * j + 0];
            t = t + a[1 * 4 + r] * view[4 * j + 1];
            t = t + a[2 * 4 + r] * view[4 * j + 2];
            t = t + a[3 * 4 + r] * view[4 * j + 3];
            proj[4 * j + r] = t;
        }
    }
}

namespace {

float sigmoid_host(float value) { return 1.0f / (1.0f + std::exp(-value)); }

}  // namespace

namespace {

void prepare_range(uint64_t first, uint64_t last, const float* opacity_raw,
                   const float* scaling_raw, const float* rotation_raw,
                   const float* specular_raw, const float* roughness_raw, float* opacity,
                   float* scaling, float* rotation, float* covariance, float* specular,
                   float* roughness) {
    for (uint64_t i = first; i < last; ++i) {
        opacity[i] = sigmoid_host(opacity_raw[i]);
        const float sx = std::exp(scaling_raw[2 * i]);
        const float sy = std::exp(scaling_raw[2 * i + 1]);
        scaling[2 * i] = sx;
        scaling[2 * i + 1] = sy;

        const float* q = rotation_raw + 4 * i;
        const float dot = (q[0] * q[0] + q[1] * q[1]) + (q[2] * q[2] + q[3] * q[3]);
        const float inv = 1.0f / std::sqrt(dot);
        const float qr = q[0] * inv, qx = q[1] * inv, qy = q[2] * inv, qz = q[3] * inv;
        rotation[4 * i + 0] = qr;
        rotation[4 * i + 1] = qx;
        rotation[4 * i + 2] = qy;
        rotation[4 * i + 3] = qz;

        // computeCov3D with modifier 1: S = diag(sx, sy, 1e-6), R from (r, x, y, z).
        float rm[3][3];  // rm[column][row]
        rm[0][0] = 1.f - 2.f * (qy * qy + qz * qz);
        rm[0][1] = 2.f * (qx * qy - qr * qz);
        rm[0][2] = 2.f * (qx * qz + qr * qy);
        rm[1][0] = 2.f * (qx * qy + qr * qz);
        rm[1][1] = 1.f - 2.f * (qx * qx + qz * qz);
        rm[1][2] = 2.f * (qy * qz - qr * qx);
        rm[2][0] = 2.f * (qx * qz - qr * qy);
        rm[2][1] = 2.f * (qy * qz + qr * qx);
        rm[2][2] = 1.f - 2.f * (qx * qx + qy * qy);
        const float s[3] = {1.0f * sx, 1.0f * sy, 0.000001f};
        // M = S * R: M[c][r] = S[0][r]*R[c][0] + S[1][r]*R[c][1] + S[2][r]*R[c][2]
        float m[3][3];
        for (int c = 0; c < 3; ++c) {
            for (int r = 0; r < 3; ++r) {
                const float s0 = r == 0 ? s[0] : 0.0f;
                const float s1 = r == 1 ? s[1] : 0.0f;
                const float s2 = r == 2 ? s[2] : 0.0f;
                float t = s0 * rm[c][0];
                t = t + s1 * rm[c][1];
                t = t + s2 * rm[c][2];
                m[c][r] = t;
            }
        }
        // Sigma = M^T * M: Sigma[c][r] = M[r][0]*M[c][0] + M[r][1]*M[c][1] + M[r][2]*M[c][2]
        auto sigma = [&](int c, int r) {
            float t = m[r][0] * m[c][0];
            t = t + m[r][1] * m[c][1];
            t = t + m[r][2] * m[c][2];
            return t;
        };
        float* out = covariance + 6 * i;
        out[0] = sigma(0, 0);
        out[1] = sigma(0, 1);
        out[2] = sigma(0, 2);
        out[3] = sigma(1, 1);
        out[4] = sigma(1, 2);
        out[5] = sigma(2, 2);
        specular[i] = sigmoid_host(specular_raw[i]);
        roughness[i] = sigmoid_host(roughness_raw[i]);
    }
}


}  // namespace

// The reference loops over the Gaussians on one thread; every Gaussian's
// arithmetic is independent, so large inputs are split into contiguous
// ranges over the host's cores with identical per-element results.
void flashgs_prepare_host(uint64_t count, const float* opacity_raw, const float* scaling_raw,
                          const float* rotation_raw, const float* specular_raw,
                          const float* roughness_raw, float* opacity, float* scaling,
                          float* rotation, float* covariance, float* specular,
                          float* roughness) {
    constexpr uint64_t kPerThread = 1u << 16;
    const unsigned cores = std::max(1u, std::thread::hardware_concurrency());
    const uint64_t wanted = (count + kPerThread - 1) / kPerThread;
    const unsigned threads = static_cast<unsigned>(std::min<uint64_t>(wanted, std::min(cores, 32u)));
    if (threads <= 1) {
        prepare_range(0, count, opacity_raw, scaling_raw, rotation_raw, specular_raw, roughness_raw,
                      opacity, scaling, rotation, covariance, specular, roughness);
        return;
    }
    std::vector<std::thread> pool;
    pool.reserve(threads);
    const uint64_t chunk = (count + threads - 1) / threads;
    for (unsigned t = 0; t < threads; ++t) {
        const uint64_t first = t * chunk, last = std::min(count, first + chunk);
        if (first >= last) break;
        try {
            pool.emplace_back(prepare_range, first, last, opacity_raw, scaling_raw, rotation_raw,
                              specular_raw, roughness_raw, opacity, scaling, rotation, covariance,
                              specular, roughness);
        } catch (...) {  // no thread available: this range on the calling thread
            prepare_range(first, last, opacity_raw, scaling_raw, rotation_raw, specular_raw,
                          roughness_raw, opacity, scaling, rotation, covariance, specular,
                          roughness);
        }
    }
    for (auto& th : pool) th.join();
}
}  // namespace hs
