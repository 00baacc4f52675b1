// Exported C ABI (include/hybridsplat_rasterizer_c_api.h).
//
// Argument validation order, status codes and message texts follow the
// reference entry points (rasterizer/c_api.cpp:129-397 for the error
// plumbing, :543-1134 for the renderer entry points, :1136-1910 for the
// elementwise and math helpers), so callers observe the same behaviour for
// invalid input. Every entry point catches C++ exceptions (guard).
#include "hybridsplat_rasterizer_c_api.h"
#include "hybridsplat_b200_ext.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusolverDn.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <exception>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "context.h"
#include "postprocess.h"
#include "view.h"
#include "pair_check.h"
#include "precise.h"

namespace hs {
cudaError_t standard_forward_noalloc(int32_t device, int32_t point_count,
                                    const float* background5, int32_t width, int32_t height,
                                    const float* means3d, const float* colors5,
                                    const float* opacities, const float* scales2,
                                    float scale_modifier, const float* rotations4,
                                    const float* viewmatrix4x4, const float* projmatrix4x4,
                                    bool prefiltered, float* output_color5, float* output_aux7,
                                    float* output_weight, int32_t* output_radii,
                                    int32_t* output_rendered, char* limit_text,
                                    uint64_t limit_capacity);
void flashgs_prepare_host(uint64_t count, const float* opacity_raw, const float* scaling_raw,
                          const float* rotation_raw, const float* specular_raw,
                          const float* roughness_raw, float* opacity, float* scaling,
                          float* rotation, float* covariance, float* specular, float* roughness);
}

namespace {

constexpr uint64_t kMathWorkspaceBytes = 2ull * 1024ull * 1024ull;
constexpr uint64_t kMathCameraOffset = 0;
constexpr uint64_t kMathIdentity3Offset = 256;
constexpr uint64_t kMathIdentity4Offset = 384;
constexpr uint64_t kMathFactorOffset = 512;
constexpr uint64_t kMathRhsOffset = 768;
constexpr uint64_t kMathPivotsOffset = 1024;
constexpr uint64_t kMathInfoOffset = 1280;
constexpr uint64_t kMathFactorArrayOffset = 1536;
constexpr uint64_t kMathRhsArrayOffset = 1792;
constexpr uint64_t kMathSolverWorkspaceOffset = 2048;
// Region of the view-camera entry (hs_b200_postprocess_camera_f32_v1), so
// that it may run on a caller's stream beside the legacy-stream helpers: its
// own inverse buffers at the offsets above relative to kMathViewOffset, and
// K, world_view^T and the camera-to-world matrix in the first 256 bytes.
constexpr uint64_t kMathViewOffset = 1024 * 1024;
constexpr uint64_t kMathViewK = kMathViewOffset;
constexpr uint64_t kMathViewWt = kMathViewOffset + 64;
constexpr uint64_t kMathViewC2w = kMathViewOffset + 128;
constexpr uint64_t kMathViewRays = kMathViewOffset + 256;  // 64 floats: rays of images under 8 pixels

unsigned char* math_at(HsRasterizerContext* c, uint64_t offset) {
    return static_cast<unsigned char*>(c->math_workspace) + offset;
}

void write_text(char* destination, uint64_t capacity, const char* text) noexcept {
    if (destination == nullptr || capacity == 0) return;
    const char* source = text == nullptr ? "" : text;
    const size_t n = std::min(std::strlen(source), static_cast<size_t>(capacity - 1));
    if (n != 0) std::memcpy(destination, source, n);
    destination[n] = '\0';
}

int32_t ok(char* error_text, uint64_t error_capacity) noexcept {
    write_text(error_text, error_capacity, "");
    return HS_STATUS_OK;
}

int32_t fail(HsStatus status, const std::string& message, char* error_text,
             uint64_t error_capacity) noexcept {
    write_text(error_text, error_capacity, message.c_str());
    return static_cast<int32_t>(status);
}

int32_t cuda_failure(cudaError_t error, const char* operation, char* error_text,
                     uint64_t error_capacity) noexcept {
    const HsStatus status =
        error == cudaErrorMemoryAllocation ? HS_STATUS_OUT_OF_MEMORY : HS_STATUS_CUDA_ERROR;
    std::string message(operation);
    message += ": ";
    if (error == hs::kWaitGaveUp) {
        message += "a bounded device wait gave up (a sort or scan look-back, or a bulk copy, "
                   "did not complete within its limit); the outputs of this call are invalid";
    } else {
        message += cudaGetErrorString(error);
    }
    return fail(status, message, error_text, error_capacity);
}

// Makes `device` current for the lifetime of the guard and restores the
// caller's current device afterwards (entry points without a handle must not
// change the device later allocations of the caller land on).
class DeviceGuard {
public:
    DeviceGuard() { had_ = cudaGetDevice(&previous_) == cudaSuccess; }
    cudaError_t select(int device) { return cudaSetDevice(device); }
    ~DeviceGuard() {
        if (had_) cudaSetDevice(previous_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int previous_ = 0;
    bool had_ = false;
};

int32_t cublas_failure(cublasStatus_t status, const char* operation, char* error_text,
                       uint64_t error_capacity) noexcept {
    std::string message(operation);
    message += ": ";
    message += cublasGetStatusString(status);
    return fail(HS_STATUS_CUDA_ERROR, message, error_text, error_capacity);
}

int32_t cusolver_failure(cusolverStatus_t status, const char* operation, char* error_text,
                         uint64_t error_capacity) noexcept {
    char message[256] = {};
    std::snprintf(message, sizeof(message), "%s: cuSOLVER status %d", operation,
                  static_cast<int>(status));
    return fail(status == CUSOLVER_STATUS_ALLOC_FAILED ? HS_STATUS_OUT_OF_MEMORY
                                                       : HS_STATUS_CUDA_ERROR,
                message, error_text, error_capacity);
}

int32_t select_device(HsRasterizerHandle handle, char* error_text,
                      uint64_t error_capacity) noexcept {
    if (handle == nullptr) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "handle is null", error_text, error_capacity);
    }
    const cudaError_t error = cudaSetDevice(handle->device);
    if (error != cudaSuccess) return cuda_failure(error, "cudaSetDevice", error_text, error_capacity);
    return HS_STATUS_OK;
}

template <typename Function>
int32_t guard(char* error_text, uint64_t error_capacity, Function&& function) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    try {
        return function();
    } catch (const std::bad_alloc& e) {
        return fail(HS_STATUS_OUT_OF_MEMORY, e.what(), error_text, error_capacity);
    } catch (const std::exception& e) {
        return fail(HS_STATUS_INTERNAL_ERROR, e.what(), error_text, error_capacity);
    } catch (...) {
        return fail(HS_STATUS_INTERNAL_ERROR, "unknown native exception", error_text,
                    error_capacity);
    }
}

cudaError_t release_math(HsRasterizerContext* c) noexcept {
    cudaError_t first = cudaSuccess;
    if (c->view_camera_event != nullptr) {
        const cudaError_t e = cudaEventDestroy(c->view_camera_event);
        if (first == cudaSuccess) first = e;
        c->view_camera_event = nullptr;
    }
    if (c->math_workspace != nullptr) {
        const cudaError_t e = cudaFree(c->math_workspace);
        if (first == cudaSuccess) first = e;
        c->math_workspace = nullptr;
    }
    for (cublasHandle_t* h : {&c->math_tf32_blas, &c->math_default_blas}) {
        if (*h != nullptr) {
            if (cublasDestroy(*h) != CUBLAS_STATUS_SUCCESS && first == cudaSuccess)
                first = cudaErrorUnknown;
            *h = nullptr;
        }
    }
    if (c->math_solver != nullptr) {
        if (cusolverDnDestroy(c->math_solver) != CUSOLVER_STATUS_SUCCESS && first == cudaSuccess)
            first = cudaErrorUnknown;
        c->math_solver = nullptr;
    }
    c->math_workspace_bytes = 0;
    return first;
}

// Persistent cuBLAS/cuSOLVER resources for the camera helpers
// (reference c_api.cpp:234-364).
int32_t initialize_math(HsRasterizerContext* c, char* error_text, uint64_t error_capacity) {
    cublasStatus_t bs = cublasCreate(&c->math_tf32_blas);
    if (bs != CUBLAS_STATUS_SUCCESS)
        return cublas_failure(bs, "math TF32 cublasCreate", error_text, error_capacity);
    ++c->math_handle_create_count;
    bs = cublasSetStream(c->math_tf32_blas, nullptr);
    if (bs == CUBLAS_STATUS_SUCCESS) bs = cublasSetPointerMode(c->math_tf32_blas, CUBLAS_POINTER_MODE_HOST);
    if (bs == CUBLAS_STATUS_SUCCESS) bs = cublasSetMathMode(c->math_tf32_blas, CUBLAS_TF32_TENSOR_OP_MATH);
    if (bs != CUBLAS_STATUS_SUCCESS)
        return cublas_failure(bs, "math TF32 handle setup", error_text, error_capacity);
    bs = cublasCreate(&c->math_default_blas);
    if (bs != CUBLAS_STATUS_SUCCESS)
        return cublas_failure(bs, "math FP32 cublasCreate", error_text, error_capacity);
    ++c->math_handle_create_count;
    bs = cublasSetStream(c->math_default_blas, nullptr);
    if (bs == CUBLAS_STATUS_SUCCESS) bs = cublasSetPointerMode(c->math_default_blas, CUBLAS_POINTER_MODE_HOST);
    if (bs == CUBLAS_STATUS_SUCCESS) bs = cublasSetMathMode(c->math_default_blas, CUBLAS_DEFAULT_MATH);
    if (bs != CUBLAS_STATUS_SUCCESS)
        return cublas_failure(bs, "math FP32 handle setup", error_text, error_capacity);
    cusolverStatus_t ss = cusolverDnCreate(&c->math_solver);
    if (ss != CUSOLVER_STATUS_SUCCESS)
        return cusolver_failure(ss, "math cusolverDnCreate", error_text, error_capacity);
    ++c->math_handle_create_count;
    ss = cusolverDnSetStream(c->math_solver, nullptr);
    if (ss != CUSOLVER_STATUS_SUCCESS)
        return cusolver_failure(ss, "math cusolverDnSetStream", error_text, error_capacity);
    cudaError_t cs = cudaMalloc(&c->math_workspace, kMathWorkspaceBytes);
    if (cs != cudaSuccess)
        return cuda_failure(cs, "math workspace cudaMalloc", error_text, error_capacity);
    c->math_workspace_bytes = kMathWorkspaceBytes;
    c->math_peak_bytes = kMathWorkspaceBytes;
    ++c->math_growth_count;
    float identity3[9] = {}, identity4[16] = {};
    for (int i = 0; i < 3; ++i) identity3[4 * i] = 1.0f;
    for (int i = 0; i < 4; ++i) identity4[5 * i] = 1.0f;
    float* factor = reinterpret_cast<float*>(math_at(c, kMathFactorOffset));
    float* rhs = reinterpret_cast<float*>(math_at(c, kMathRhsOffset));
    cs = cudaMemcpy(math_at(c, kMathIdentity3Offset), identity3, sizeof(identity3), cudaMemcpyHostToDevice);
    if (cs == cudaSuccess)
        cs = cudaMemcpy(math_at(c, kMathIdentity4Offset), identity4, sizeof(identity4), cudaMemcpyHostToDevice);
    if (cs == cudaSuccess)
        cs = cudaMemcpy(math_at(c, kMathFactorArrayOffset), &factor, sizeof(factor), cudaMemcpyHostToDevice);
    if (cs == cudaSuccess)
        cs = cudaMemcpy(math_at(c, kMathRhsArrayOffset), &rhs, sizeof(rhs), cudaMemcpyHostToDevice);
    float* view_factor = reinterpret_cast<float*>(math_at(c, kMathViewOffset + kMathFactorOffset));
    float* view_rhs = reinterpret_cast<float*>(math_at(c, kMathViewOffset + kMathRhsOffset));
    if (cs == cudaSuccess)
        cs = cudaMemcpy(math_at(c, kMathViewOffset + kMathFactorArrayOffset), &view_factor, sizeof(view_factor),
                        cudaMemcpyHostToDevice);
    if (cs == cudaSuccess)
        cs = cudaMemcpy(math_at(c, kMathViewOffset + kMathRhsArrayOffset), &view_rhs, sizeof(view_rhs),
                        cudaMemcpyHostToDevice);
    if (cs != cudaSuccess)
        return cuda_failure(cs, "math workspace initialization", error_text, error_capacity);
    ss = cusolverDnSgetrf_bufferSize(c->math_solver, 4, 4, factor, 4, &c->math_inverse_workspace_count);
    if (ss != CUSOLVER_STATUS_SUCCESS)
        return cusolver_failure(ss, "math inverse workspace query", error_text, error_capacity);
    if (kMathViewOffset + kMathSolverWorkspaceOffset + uint64_t(c->math_inverse_workspace_count) * sizeof(float) >
        kMathWorkspaceBytes) {
        return fail(HS_STATUS_RANGE_ERROR, "math inverse workspace exceeds persistent allocation",
                    error_text, error_capacity);
    }
    return HS_STATUS_OK;
}

bool finite3(const float* v) {
    return std::isfinite(v[0]) && std::isfinite(v[1]) && std::isfinite(v[2]);
}

// Guards the elementwise entry points: count == 0 succeeds with NULL buffers.
template <class Launch>
int32_t elementwise(const char* name, uint64_t count, bool buffers_present, char* error_text,
                    uint64_t error_capacity, Launch&& launch) {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (count == 0) return ok(error_text, error_capacity);
        if (!buffers_present) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        std::string(name) + " received a null non-empty buffer", error_text,
                        error_capacity);
        }
        const cudaError_t e = launch();
        if (e != cudaSuccess)
            return cuda_failure(e, (std::string(name) + " launch").c_str(), error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

}  // namespace

namespace {

// Checks one FlashGS call as hs_flashgs_forward_f32_v1 does and converts it
// (the host camera and background are copied).
int32_t check_flashgs(const HsB200FlashgsCallV2& a, hs::FlashgsCall* call, char* error_text,
                      uint64_t error_capacity) {
    if (a.handle == nullptr || a.camera_position3 == nullptr || a.camera_rotation9 == nullptr ||
        a.background3 == nullptr || a.output_color3 == nullptr || a.output_other2 == nullptr ||
        a.output_depth1 == nullptr || a.output_alpha1 == nullptr || a.output_normal3 == nullptr ||
        a.output_median_depth1 == nullptr || a.output_distortion1 == nullptr ||
        a.output_num_rendered == nullptr) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS received a null required handle or buffer",
                    error_text, error_capacity);
    }
    if (a.point_count > static_cast<uint64_t>(INT_MAX) || a.width <= 0 || a.height <= 0 ||
        (a.use_sh != 0 && a.use_sh != 1) || a.initial_pair_capacity == 0 ||
        a.initial_pair_capacity > static_cast<uint64_t>(INT_MAX) ||
        !std::isfinite(a.scale_modifier) || a.scale_modifier <= 0.0f ||
        !std::isfinite(a.focal_x) || a.focal_x <= 0.0f || !std::isfinite(a.focal_y) ||
        a.focal_y <= 0.0f || !std::isfinite(a.z_near) || a.z_near <= 0.0f ||
        !std::isfinite(a.z_far) || a.z_far <= a.z_near) {
        return fail(HS_STATUS_RANGE_ERROR, "FlashGS dimensions or scalar arguments are invalid",
                    error_text, error_capacity);
    }
    if (!finite3(a.camera_position3) || !finite3(a.background3)) {
        return fail(HS_STATUS_RANGE_ERROR, "FlashGS camera position or background is not finite",
                    error_text, error_capacity);
    }
    for (int i = 0; i < 9; ++i) {
        if (!std::isfinite(a.camera_rotation9[i])) {
            return fail(HS_STATUS_RANGE_ERROR, "FlashGS camera rotation is not finite", error_text,
                        error_capacity);
        }
    }
    if (a.point_count != 0 &&
        (a.positions3 == nullptr || a.opacities1 == nullptr || a.covariance6 == nullptr ||
         a.scales2 == nullptr || a.rotations4 == nullptr || a.specular1 == nullptr ||
         a.roughness1 == nullptr || (a.use_sh != 0 && a.shs48 == nullptr) ||
         (a.use_sh == 0 && a.colors3 == nullptr))) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "non-empty FlashGS input contains a null buffer",
                    error_text, error_capacity);
    }
    const uint32_t grid_y = static_cast<uint32_t>((a.height + 15) / 16);
    if (a.tile_row_begin >= a.tile_row_end ||
        (a.tile_row_end != UINT32_MAX && a.tile_row_end > grid_y)) {
        return fail(HS_STATUS_RANGE_ERROR, "tile rows must satisfy 0 <= begin < end <= tile rows",
                    error_text, error_capacity);
    }
    hs::FlashgsCall& c = *call;
    c.point_count = static_cast<int32_t>(a.point_count);
    c.width = a.width;
    c.height = a.height;
    c.positions3 = a.positions3;
    c.shs48 = a.shs48;
    c.colors3 = a.colors3;
    c.use_sh = a.use_sh != 0;
    c.opacities1 = a.opacities1;
    c.covariance6 = a.covariance6;
    c.scales2 = a.scales2;
    c.scale_modifier = a.scale_modifier;
    c.rotations4 = a.rotations4;
    c.specular1 = a.specular1;
    c.roughness1 = a.roughness1;
    std::memcpy(c.camera_position3, a.camera_position3, sizeof(c.camera_position3));
    std::memcpy(c.camera_rotation9, a.camera_rotation9, sizeof(c.camera_rotation9));
    c.focal_x = a.focal_x;
    c.focal_y = a.focal_y;
    c.z_far = a.z_far;
    c.z_near = a.z_near;
    std::memcpy(c.background3, a.background3, sizeof(c.background3));
    c.initial_pair_capacity = a.initial_pair_capacity;
    c.output_color3 = a.output_color3;
    c.output_other2 = a.output_other2;
    c.output_depth1 = a.output_depth1;
    c.output_alpha1 = a.output_alpha1;
    c.output_normal3 = a.output_normal3;
    c.output_median_depth1 = a.output_median_depth1;
    c.output_distortion1 = a.output_distortion1;
    c.output_num_rendered = a.output_num_rendered;
    c.stream = nullptr;
    c.row_begin = a.tile_row_begin;
    c.row_end = a.tile_row_end;
    return HS_STATUS_OK;
}

// Checks one standard call as hs_rasterizer_forward_f32_v1 does and converts it.
int32_t check_rasterizer(const HsB200RasterizerCallV2& a, hs::StandardCall* call,
                         char* error_text, uint64_t error_capacity) {
    if (a.handle == nullptr || a.background5 == nullptr || a.output_color5 == nullptr ||
        a.output_aux7 == nullptr || a.output_rendered == nullptr) {
        return fail(HS_STATUS_INVALID_ARGUMENT,
                    "rasterizer received a null required handle or buffer", error_text,
                    error_capacity);
    }
    if (a.point_count > static_cast<uint64_t>(INT_MAX) || a.width <= 0 || a.height <= 0 ||
        !std::isfinite(a.scale_modifier) || !std::isfinite(a.tan_fovx) ||
        !std::isfinite(a.tan_fovy) || a.tan_fovx <= 0.0f || a.tan_fovy <= 0.0f ||
        (a.prefiltered != 0 && a.prefiltered != 1)) {
        return fail(HS_STATUS_RANGE_ERROR, "rasterizer dimensions or scalar arguments are invalid",
                    error_text, error_capacity);
    }
    if (a.point_count != 0 &&
        (a.means3d == nullptr || a.colors5 == nullptr || a.opacities == nullptr ||
         a.scales2 == nullptr || a.rotations4 == nullptr || a.viewmatrix4x4 == nullptr ||
         a.projmatrix4x4 == nullptr || a.camera_position3 == nullptr ||
         a.output_weight == nullptr || a.output_radii == nullptr)) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "non-empty rasterizer input contains a null buffer",
                    error_text, error_capacity);
    }
    const uint32_t grid_y = static_cast<uint32_t>((a.height + 15) / 16);
    if (a.tile_row_begin >= a.tile_row_end ||
        (a.tile_row_end != UINT32_MAX && a.tile_row_end > grid_y)) {
        return fail(HS_STATUS_RANGE_ERROR, "tile rows must satisfy 0 <= begin < end <= tile rows",
                    error_text, error_capacity);
    }
    hs::StandardCall& c = *call;
    c.point_count = static_cast<int32_t>(a.point_count);
    c.background5 = a.background5;
    c.width = a.width;
    c.height = a.height;
    c.means3d = a.means3d;
    c.colors5 = a.colors5;
    c.opacities = a.opacities;
    c.scales2 = a.scales2;
    c.scale_modifier = a.scale_modifier;
    c.rotations4 = a.rotations4;
    c.viewmatrix4x4 = a.viewmatrix4x4;
    c.projmatrix4x4 = a.projmatrix4x4;
    c.camera_position3 = a.camera_position3;
    c.tan_fovx = a.tan_fovx;
    c.tan_fovy = a.tan_fovy;
    c.prefiltered = a.prefiltered != 0;
    c.output_color5 = a.output_color5;
    c.output_aux7 = a.output_aux7;
    c.output_weight = a.output_weight;
    c.output_radii = a.output_radii;
    c.output_rendered = a.output_rendered;
    c.stream = nullptr;
    c.row_begin = a.tile_row_begin;
    c.row_end = a.tile_row_end;
    return HS_STATUS_OK;
}

HsB200FlashgsCallV2 flashgs_args(
    HsRasterizerHandle handle, uint64_t point_count, int32_t width, int32_t height,
    const float* positions3, const float* shs48, const float* colors3, int32_t use_sh,
    const float* opacities1, const float* covariance6, const float* scales2, float scale_modifier,
    const float* rotations4, const float* specular1, const float* roughness1,
    const float* camera_position3, const float* camera_rotation9, float focal_x, float focal_y,
    float z_far, float z_near, const float* background3, uint64_t initial_pair_capacity,
    float* output_color3, float* output_other2, float* output_depth1, float* output_alpha1,
    float* output_normal3, float* output_median_depth1, float* output_distortion1,
    int32_t* output_num_rendered) {
    HsB200FlashgsCallV2 a{};
    a.handle = handle;
    a.point_count = point_count;
    a.width = width;
    a.height = height;
    a.positions3 = positions3;
    a.shs48 = shs48;
    a.colors3 = colors3;
    a.use_sh = use_sh;
    a.scale_modifier = scale_modifier;
    a.opacities1 = opacities1;
    a.covariance6 = covariance6;
    a.scales2 = scales2;
    a.rotations4 = rotations4;
    a.specular1 = specular1;
    a.roughness1 = roughness1;
    a.camera_position3 = camera_position3;
    a.camera_rotation9 = camera_rotation9;
    a.focal_x = focal_x;
    a.focal_y = focal_y;
    a.z_far = z_far;
    a.z_near = z_near;
    a.background3 = background3;
    a.initial_pair_capacity = initial_pair_capacity;
    a.output_color3 = output_color3;
    a.output_other2 = output_other2;
    a.output_depth1 = output_depth1;
    a.output_alpha1 = output_alpha1;
    a.output_normal3 = output_normal3;
    a.output_median_depth1 = output_median_depth1;
    a.output_distortion1 = output_distortion1;
    a.output_num_rendered = output_num_rendered;
    a.tile_row_begin = 0;
    a.tile_row_end = UINT32_MAX;
    return a;
}

HsB200RasterizerCallV2 rasterizer_args(
    HsRasterizerHandle handle, uint64_t point_count, const float* background5, int32_t width,
    int32_t height, const float* means3d, const float* colors5, const float* opacities,
    const float* scales2, float scale_modifier, const float* rotations4,
    const float* viewmatrix4x4, const float* projmatrix4x4, const float* camera_position3,
    float tan_fovx, float tan_fovy, int32_t prefiltered, float* output_color5, float* output_aux7,
    float* output_weight, int32_t* output_radii, int32_t* output_rendered) {
    HsB200RasterizerCallV2 a{};
    a.handle = handle;
    a.point_count = point_count;
    a.background5 = background5;
    a.width = width;
    a.height = height;
    a.means3d = means3d;
    a.colors5 = colors5;
    a.opacities = opacities;
    a.scales2 = scales2;
    a.scale_modifier = scale_modifier;
    a.prefiltered = prefiltered;
    a.rotations4 = rotations4;
    a.viewmatrix4x4 = viewmatrix4x4;
    a.projmatrix4x4 = projmatrix4x4;
    a.camera_position3 = camera_position3;
    a.tan_fovx = tan_fovx;
    a.tan_fovy = tan_fovy;
    a.output_color5 = output_color5;
    a.output_aux7 = output_aux7;
    a.output_weight = output_weight;
    a.output_radii = output_radii;
    a.output_rendered = output_rendered;
    a.tile_row_begin = 0;
    a.tile_row_end = UINT32_MAX;
    return a;
}

int32_t flashgs_entry(const HsB200FlashgsCallV2& a, char* error_text,
                      uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        hs::FlashgsCall call;
        const int32_t cs = check_flashgs(a, &call, error_text, error_capacity);
        if (cs != HS_STATUS_OK) return cs;
        const int32_t ds = select_device(a.handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(a.handle->mutex);
        const cudaError_t e = hs::flashgs_forward(a.handle, call);
        if (e != cudaSuccess)
            return cuda_failure(e, "deterministic FlashGS forward", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t rasterizer_entry(const HsB200RasterizerCallV2& a, char* error_text,
                         uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        hs::StandardCall call;
        const int32_t cs = check_rasterizer(a, &call, error_text, error_capacity);
        if (cs != HS_STATUS_OK) return cs;
        const int32_t ds = select_device(a.handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(a.handle->mutex);
        const cudaError_t e = hs::standard_forward(a.handle, call);
        if (e != cudaSuccess)
            return cuda_failure(e, "five-channel rasterizer forward", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

// Shared body of the forward_many entry points: checks every call before
// anything is queued, requires distinct handles on one device, locks the
// handles in address order and runs the calls concurrently.
template <class Args, class Call, class Check, class Run>
int32_t many_entry(const Args* calls, uint32_t call_count, void* stream, const char* what,
                   Check&& check, Run&& run, char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (calls == nullptr && call_count != 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "calls is null", error_text, error_capacity);
        }
        if (call_count == 0) return ok(error_text, error_capacity);
        std::vector<Call> converted(call_count);
        std::vector<HsRasterizerContext*> contexts(call_count);
        for (uint32_t i = 0; i < call_count; ++i) {
            const int32_t cs = check(calls[i], &converted[i], error_text, error_capacity);
            if (cs != HS_STATUS_OK) return cs;
            contexts[i] = calls[i].handle;
        }
        for (uint32_t i = 0; i < call_count; ++i) {
            if (contexts[i]->device != contexts[0]->device) {
                return fail(HS_STATUS_INVALID_ARGUMENT, "all calls must use handles of one device",
                            error_text, error_capacity);
            }
        }
        std::vector<HsRasterizerContext*> lock_order = contexts;
        std::sort(lock_order.begin(), lock_order.end());
        if (std::adjacent_find(lock_order.begin(), lock_order.end()) != lock_order.end()) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "each call needs its own handle", error_text,
                        error_capacity);
        }
        const int32_t ds = select_device(contexts[0], error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::vector<std::unique_lock<std::mutex>> locks;
        locks.reserve(call_count);
        for (HsRasterizerContext* c : lock_order) locks.emplace_back(c->mutex);
        const cudaError_t e = run(contexts.data(), converted.data(), call_count,
                                  static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_failure(e, what, error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

// The trace section shared by the one-view entries (fields of the same
// names in HsB200StandardViewV2 and HsB200FlashgsViewV2): the checks of
// hs_optix_trace_f32_v1 on its arguments, and the call itself.
template <class View>
int32_t check_view_trace(const View& v, uint64_t rays, const float* shs, const float* others, const char* what,
                         char* error_text, uint64_t error_capacity) {
    if (v.trace != 0 && v.trace != 1) {
        return fail(HS_STATUS_RANGE_ERROR, std::string(what) + " trace must be 0 or 1", error_text,
                    error_capacity);
    }
    if (v.trace == 0) return HS_STATUS_OK;
    if (v.trace_coefficients == 0 || v.trace_coefficients > 16 || v.trace_degree > 3 ||
        v.trace_coefficients < (v.trace_degree + 1) * (v.trace_degree + 1) ||
        (v.use_others != 0 && v.use_others != 1) || v.max_trace_depth < 0 || v.max_trace_depth > 1 ||
        !std::isfinite(v.specular_threshold) || rays > UINT32_MAX) {
        return fail(HS_STATUS_RANGE_ERROR, "OptiX trace dimensions or scalars are invalid", error_text,
                    error_capacity);
    }
    if (rays != 0 && (v.reflection_ray_origins3 == nullptr || v.reflection_ray_directions3 == nullptr ||
                      v.trace_background3 == nullptr || shs == nullptr || others == nullptr ||
                      v.trace_rgb3 == nullptr || v.trace_depth1 == nullptr || v.trace_acc1 == nullptr ||
                      v.trace_normal3 == nullptr || v.trace_dist1 == nullptr || v.trace_aux2 == nullptr ||
                      v.trace_mid32 == nullptr || v.trace_wet1 == nullptr)) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX trace received a null non-empty buffer", error_text,
                    error_capacity);
    }
    return HS_STATUS_OK;
}

// hs_optix_trace_f32_v1 of a view: scale modifier 1, start_from_first 0, the
// rays of the view's reflection preparation (renderer.py:281-301, 385-405).
template <class View>
hs::TraceCall view_trace_call(const View& v, uint64_t rays, const float* means3d, const float* shs,
                              const float* others, const float* opacities, const float* scales2,
                              const float* rotations4, const float* view4x4, const float* proj4x4,
                              const float* center3, cudaStream_t stream) {
    hs::TraceCall t;
    t.ray_count = rays;
    t.ray_origins3 = v.reflection_ray_origins3;
    t.ray_directions3 = v.reflection_ray_directions3;
    t.background3 = v.trace_background3;
    t.means3d = means3d;
    t.shs_m3 = shs;
    t.coefficient_count = v.trace_coefficients;
    t.degree = v.trace_degree;
    t.others2 = others;
    t.opacities = opacities;
    t.scales2 = scales2;
    t.scale_modifier = 1.0f;
    t.rotations4 = rotations4;
    t.viewmatrix4x4 = view4x4;
    t.projmatrix4x4 = proj4x4;
    t.camera_position3 = center3;
    t.start_from_first = 0;
    t.max_trace_depth = v.max_trace_depth;
    t.specular_threshold = v.specular_threshold;
    t.use_others = v.use_others;
    t.output_rgb3 = v.trace_rgb3;
    t.output_depth1 = v.trace_depth1;
    t.output_acc1 = v.trace_acc1;
    t.output_normal3 = v.trace_normal3;
    t.output_dist1 = v.trace_dist1;
    t.output_aux2 = v.trace_aux2;
    t.output_mid32 = v.trace_mid32;
    t.output_wet1 = v.trace_wet1;
    t.stream = stream;
    return t;
}

// ---- graph replays of the one-view entries ----

constexpr size_t kMaxViewGraphs = 4;

// HS_B200_VIEW_GRAPHS=0 turns the replays off (every view queued directly).
bool view_graphs_enabled() {
    const char* flag = std::getenv("HS_B200_VIEW_GRAPHS");
    return flag == nullptr || std::strcmp(flag, "0") != 0;
}

template <class T>
void key_put(std::vector<unsigned char>& key, const T& value) {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&value);
    key.insert(key.end(), p, p + sizeof(T));
}

// What a captured view depends on: the entry's argument block (every pointer,
// size, scalar and the stream) and, per context, the buffers the graph reads
// and writes (their addresses and sizes).
std::vector<unsigned char> view_graph_key(const void* args, size_t bytes, HsRasterizerContext* const* contexts,
                                          uint32_t count) {
    const unsigned char* a = static_cast<const unsigned char*>(args);
    std::vector<unsigned char> key(a, a + bytes);
    for (uint32_t i = 0; i < count; ++i) {
        const HsRasterizerContext* c = contexts[i];
        key_put(key, c);
        for (const hs::DeviceBuffer* b : {&c->std_geometry, &c->std_image, &c->std_binning, &c->fg_gaussian,
                                          &c->fg_pairs, &c->fg_sort, &c->fg_ranges}) {
            key_put(key, b->ptr);
            key_put(key, b->bytes);
        }
        key_put(key, c->std_total_mapped);
        key_put(key, c->fg_total_mapped);
        key_put(key, c->device_error);
        key_put(key, c->side_stream);
        key_put(key, c->math_workspace);
        key_put(key, c->math_workspace_bytes);
    }
    return key;
}

HsRasterizerContext::ViewGraph* find_view_graph(HsRasterizerContext* c, const std::vector<unsigned char>& key) {
    for (HsRasterizerContext::ViewGraph& g : c->view_graphs) {
        if (g.key == key) return &g;
    }
    return nullptr;
}

// Keeps at most kMaxViewGraphs, dropping the least recently used (an
// executable still in flight is freed when it completes).
HsRasterizerContext::ViewGraph* insert_view_graph(HsRasterizerContext* c, std::vector<unsigned char> key,
                                                  cudaGraphExec_t exec, const uint32_t* capacity) {
    if (c->view_graphs.size() >= kMaxViewGraphs) {
        auto oldest = std::min_element(c->view_graphs.begin(), c->view_graphs.end(),
                                       [](const auto& x, const auto& y) { return x.last_use < y.last_use; });
        if (oldest->exec != nullptr) cudaGraphExecDestroy(oldest->exec);
        c->view_graphs.erase(oldest);
    }
    HsRasterizerContext::ViewGraph g;
    g.key = std::move(key);
    g.exec = exec;
    g.capacity[0] = capacity[0];
    g.capacity[1] = capacity[1];
    g.last_use = ++c->view_graph_clock;
    c->view_graphs.push_back(std::move(g));
    return &c->view_graphs.back();
}

// Captures queue(true) on `stream` into an uploaded executable graph; null
// when the capture or the instantiation fails (the view then runs directly).
// After a failed queue every branch stream is joined back so that the
// capture can end.
template <class Queue>
cudaGraphExec_t capture_view(cudaStream_t stream, const Queue& queue, std::initializer_list<cudaStream_t> branches,
                             cudaEvent_t join_event) {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    const bool queued = queue();
    if (!queued) {
        for (cudaStream_t b : branches) {
            if (b != nullptr && cudaEventRecord(join_event, b) == cudaSuccess)
                (void)cudaStreamWaitEvent(stream, join_event, 0);
        }
    }
    const cudaError_t end = cudaStreamEndCapture(stream, &graph);
    if (queued && end == cudaSuccess && graph != nullptr) {
        if (cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
            exec = nullptr;
        } else if (cudaGraphUpload(exec, stream) != cudaSuccess) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
    }
    if (graph != nullptr) cudaGraphDestroy(graph);
    (void)cudaGetLastError();
    return exec;
}

}  // namespace

extern "C" {

uint32_t hs_rasterizer_abi_version(void) noexcept { return HS_RASTERIZER_ABI_VERSION; }

int32_t hs_rasterizer_build_info(char* output_text, uint64_t output_capacity) noexcept {
    if (output_text == nullptr || output_capacity == 0) return HS_STATUS_INVALID_ARGUMENT;
    const char* info =
        "{\"abi\":2,\"build_id\":\"hybridsplat-b200\",\"cuda\":\"12.9\",\"sm\":100,"
        "\"arch\":\"sm_100a\",\"cxx_standard\":17,\"cuda_standard\":17,"
        "\"fast_math\":false,\"stream\":0,"
        "\"flashgs_forward\":\"deterministic_depth_then_tile_sort_v1\","
        "\"flashgs_preprocess_invisible_slots\":\"zero\","
        "\"five_channel_rasterizer\":\"forward_v1\","
        "\"optix_reflection_tracer\":\"cuda_bvh_v1\","
        "\"workspace_growth\":\"1.25x_align_2mib\"}";
    write_text(output_text, output_capacity, info);
    return std::strlen(info) + 1 > output_capacity ? HS_STATUS_RANGE_ERROR : HS_STATUS_OK;
}

int32_t hs_rasterizer_create(int32_t device, HsRasterizerHandle* handle, char* error_text,
                             uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "handle output is null", error_text, error_capacity);
        }
        *handle = nullptr;
        int device_count = 0;
        cudaError_t e = cudaGetDeviceCount(&device_count);
        if (e != cudaSuccess) return cuda_failure(e, "cudaGetDeviceCount", error_text, error_capacity);
        if (device < 0 || device >= device_count) {
            return fail(HS_STATUS_RANGE_ERROR, "device is outside the visible CUDA device range",
                        error_text, error_capacity);
        }
        e = cudaSetDevice(device);
        if (e != cudaSuccess) return cuda_failure(e, "cudaSetDevice", error_text, error_capacity);
        *handle = new HsRasterizerContext(device);
        const int32_t status = initialize_math(*handle, error_text, error_capacity);
        if (status != HS_STATUS_OK) {
            release_math(*handle);
            delete *handle;
            *handle = nullptr;
            return status;
        }
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_synchronize(HsRasterizerHandle handle, char* error_text,
                                  uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        const cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_failure(e, "cudaDeviceSynchronize", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_workspace_stats(HsRasterizerHandle handle,
                                      HsRasterizerWorkspaceStatsV1* stats, char* error_text,
                                      uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr || stats == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "handle or stats is null", error_text, error_capacity);
        }
        if (stats->struct_size != sizeof(HsRasterizerWorkspaceStatsV1) ||
            stats->abi_version != HS_RASTERIZER_ABI_VERSION) {
            return fail(HS_STATUS_ABI_MISMATCH, "workspace stats ABI does not match", error_text,
                        error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        stats->device = handle->device;
        stats->reserved = 0;
        stats->geometry_bytes = handle->std_geometry.bytes;
        stats->binning_bytes = handle->std_binning.bytes;
        stats->image_bytes = handle->std_image.bytes;
        stats->current_bytes = hs::standard_current_bytes(handle);
        stats->peak_bytes = handle->std_peak_bytes;
        stats->growth_count = handle->std_growth_count;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_release_workspace(HsRasterizerHandle handle, char* error_text,
                                        uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_failure(e, "cudaDeviceSynchronize", error_text, error_capacity);
        e = hs::standard_release(handle);
        if (e != cudaSuccess) return cuda_failure(e, "release rasterizer workspace", error_text, error_capacity);
        e = hs::flashgs_release(handle);
        if (e != cudaSuccess) return cuda_failure(e, "release FlashGS workspace", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_math_workspace_stats_v2(HsRasterizerHandle handle,
                                              HsMathWorkspaceStatsV2* stats, char* error_text,
                                              uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr || stats == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "handle or math stats is null", error_text,
                        error_capacity);
        }
        if (stats->struct_size != sizeof(HsMathWorkspaceStatsV2) ||
            stats->abi_version != HS_RASTERIZER_ABI_VERSION) {
            return fail(HS_STATUS_ABI_MISMATCH, "math workspace stats ABI does not match",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        stats->device = handle->device;
        stats->handles_ready = handle->math_tf32_blas != nullptr &&
                                       handle->math_default_blas != nullptr &&
                                       handle->math_solver != nullptr
                                   ? 1u
                                   : 0u;
        stats->workspace_bytes = handle->math_workspace_bytes;
        stats->current_bytes = handle->math_workspace_bytes;
        stats->peak_bytes = handle->math_peak_bytes;
        stats->growth_count = handle->math_growth_count;
        stats->handle_create_count = handle->math_handle_create_count;
        stats->camera_center_calls = handle->math_camera_center_calls;
        stats->general_inverse_calls = handle->math_general_inverse_calls;
        stats->matmul_calls = handle->math_matmul_calls;
        stats->pixel_world_calls = handle->math_pixel_world_calls;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_destroy(HsRasterizerHandle handle, char* error_text,
                              uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "handle is null", error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        {
            std::lock_guard<std::mutex> lock(handle->mutex);
            cudaError_t e = cudaDeviceSynchronize();
            if (e != cudaSuccess) return cuda_failure(e, "cudaDeviceSynchronize", error_text, error_capacity);
            e = hs::standard_release(handle);
            if (e != cudaSuccess) return cuda_failure(e, "release rasterizer workspace", error_text, error_capacity);
            e = hs::flashgs_release(handle);
            if (e != cudaSuccess) return cuda_failure(e, "release FlashGS context", error_text, error_capacity);
            e = release_math(handle);
            if (e != cudaSuccess) return cuda_failure(e, "release math context", error_text, error_capacity);
            e = hs::trace_release(handle);
            if (e != cudaSuccess) return cuda_failure(e, "release trace scene", error_text, error_capacity);
            hs::stage_timing_destroy(handle->timer);
            if (handle->std_count_event != nullptr) cudaEventDestroy(handle->std_count_event);
            if (handle->fg_count_event != nullptr) cudaEventDestroy(handle->fg_count_event);
            if (handle->device_error != nullptr) cudaFree(handle->device_error);
            hs::destroy_side_stream(handle);
        }
        delete handle;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_flashgs_forward_f32_v1(
    HsRasterizerHandle handle, uint64_t point_count, int32_t width, int32_t height,
    const float* positions3, const float* shs48, const float* colors3, int32_t use_sh,
    const float* opacities1, const float* covariance6, const float* scales2, float scale_modifier,
    const float* rotations4, const float* specular1, const float* roughness1,
    const float* camera_position3, const float* camera_rotation9, float focal_x, float focal_y,
    float z_far, float z_near, const float* background3, uint64_t initial_pair_capacity,
    float* output_color3, float* output_other2, float* output_depth1, float* output_alpha1,
    float* output_normal3, float* output_median_depth1, float* output_distortion1,
    int32_t* output_num_rendered, char* error_text, uint64_t error_capacity) noexcept {
    return flashgs_entry(
        flashgs_args(handle, point_count, width, height, positions3, shs48, colors3, use_sh,
                     opacities1, covariance6, scales2, scale_modifier, rotations4, specular1,
                     roughness1, camera_position3, camera_rotation9, focal_x, focal_y, z_far,
                     z_near, background3, initial_pair_capacity, output_color3, output_other2,
                     output_depth1, output_alpha1, output_normal3, output_median_depth1,
                     output_distortion1, output_num_rendered),
        error_text, error_capacity);
}

int32_t hs_flashgs_workspace_stats_v1(HsRasterizerHandle handle,
                                      HsFlashgsWorkspaceStatsV1* stats, char* error_text,
                                      uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr || stats == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "handle or FlashGS stats is null", error_text,
                        error_capacity);
        }
        if (stats->struct_size != sizeof(HsFlashgsWorkspaceStatsV1) ||
            stats->abi_version != HS_RASTERIZER_ABI_VERSION) {
            return fail(HS_STATUS_ABI_MISMATCH, "FlashGS workspace stats ABI does not match",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        stats->device = handle->device;
        stats->initialized = handle->fg_pairs.ptr != nullptr ? 1u : 0u;
        stats->gaussian_capacity = handle->fg_gaussian_capacity;
        stats->pair_capacity = handle->fg_pair_capacity;
        stats->range_capacity = handle->fg_range_capacity;
        stats->output_pixel_capacity = 0;
        stats->gaussian_bytes = handle->fg_gaussian.bytes;
        stats->pair_bytes = handle->fg_pairs.bytes;
        stats->cub_bytes = handle->fg_sort.bytes;
        stats->ranges_bytes = handle->fg_ranges.bytes;
        stats->output_bytes = 0;
        stats->current_bytes = hs::flashgs_current_bytes(handle);
        stats->peak_bytes = handle->fg_peak_bytes;
        stats->growth_count = handle->fg_growth_count;
        stats->overflow_retry_count = handle->fg_overflow_retry_count;
        stats->forward_calls = handle->fg_forward_calls;
        stats->last_point_count = handle->fg_last_point_count;
        stats->last_num_rendered = handle->fg_last_num_rendered;
        stats->last_tile_count = handle->fg_last_tile_count;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_flashgs_prepare_npz_host_f32_v1(uint64_t point_count, const float* opacity_raw1,
                                           const float* scaling_raw2, const float* rotation_raw4,
                                           const float* specular_raw1,
                                           const float* roughness_raw1, float* opacity1,
                                           float* scaling2, float* rotation4, float* covariance6,
                                           float* specular1, float* roughness1, char* error_text,
                                           uint64_t error_capacity) noexcept {
    // Validation order of flashgs_prepare.cpp:46-56: the error buffer is
    // cleared first, then checked.
    write_text(error_text, error_capacity, "");
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    if (point_count == 0) return HS_STATUS_OK;
    if (opacity_raw1 == nullptr || scaling_raw2 == nullptr || rotation_raw4 == nullptr ||
        specular_raw1 == nullptr || roughness_raw1 == nullptr || opacity1 == nullptr ||
        scaling2 == nullptr || rotation4 == nullptr || covariance6 == nullptr ||
        specular1 == nullptr || roughness1 == nullptr) {
        write_text(error_text, error_capacity, "FlashGS NPZ preparation received a null host buffer");
        return HS_STATUS_INVALID_ARGUMENT;
    }
    try {
        hs::flashgs_prepare_host(point_count, opacity_raw1, scaling_raw2, rotation_raw4,
                                 specular_raw1, roughness_raw1, opacity1, scaling2, rotation4,
                                 covariance6, specular1, roughness1);
        return HS_STATUS_OK;
    } catch (const std::exception& e) {
        write_text(error_text, error_capacity, e.what());
        return HS_STATUS_INTERNAL_ERROR;
    } catch (...) {
        write_text(error_text, error_capacity, "unknown FlashGS NPZ preparation error");
        return HS_STATUS_INTERNAL_ERROR;
    }
}

int32_t hs_flashgs_debug_copy_v1(HsRasterizerHandle handle, uint64_t point_capacity,
                                 uint64_t pair_capacity, uint64_t tile_capacity,
                                 float* points_xy2, float* rgb3, float* other2,
                                 float* conic_opacity4, float* normal_opacity4, float* tu3,
                                 float* tv3, float* tw3, uint64_t* sorted_keys,
                                 uint32_t* sorted_values, int32_t* tile_ranges2,
                                 char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS debug copy received a null context",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        const cudaError_t e = hs::flashgs_debug_copy(
            handle, point_capacity, pair_capacity, tile_capacity, points_xy2, rgb3, other2,
            conic_opacity4, normal_opacity4, tu3, tv3, tw3, sorted_keys, sorted_values,
            tile_ranges2);
        if (e != cudaSuccess) return cuda_failure(e, "FlashGS debug copy", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_standard_debug_copy_v1(HsRasterizerHandle handle, uint64_t point_capacity,
                                       float* points_xy2, float* transmats9,
                                       float* normal_opacity4, char* error_text,
                                       uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "standard debug copy received a null context",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        const cudaError_t e = hs::standard_debug_copy(handle, point_capacity, points_xy2,
                                                      transmats9, normal_opacity4);
        if (e != cudaSuccess) return cuda_failure(e, "standard debug copy", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_forward_f32_v1(
    HsRasterizerHandle handle, uint64_t point_count, const float* background5, int32_t width,
    int32_t height, const float* means3d, const float* colors5, const float* opacities,
    const float* scales2, float scale_modifier, const float* rotations4,
    const float* viewmatrix4x4, const float* projmatrix4x4, const float* camera_position3,
    float tan_fovx, float tan_fovy, int32_t prefiltered, float* output_color5, float* output_aux7,
    float* output_weight, int32_t* output_radii, int32_t* output_rendered, char* error_text,
    uint64_t error_capacity) noexcept {
    return rasterizer_entry(
        rasterizer_args(handle, point_count, background5, width, height, means3d, colors5,
                        opacities, scales2, scale_modifier, rotations4, viewmatrix4x4,
                        projmatrix4x4, camera_position3, tan_fovx, tan_fovy, prefiltered,
                        output_color5, output_aux7, output_weight, output_radii, output_rendered),
        error_text, error_capacity);
}

// Reflection-trace entry points (reference optix/optix_backend.cpp:375-662):
// same arguments, checks, error texts and stats; the scene is a BVH built by
// this library and the trace runs on CUDA cores (trace.cu), with no OptiX.
int32_t hs_optix_build_scene_v1(HsRasterizerHandle handle, const float* vertices3,
                                uint64_t vertex_count, const int32_t* triangles3,
                                uint64_t triangle_count, uint64_t scene_signature, int32_t rebuild,
                                int32_t* output_status, char* error_text,
                                uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr || vertices3 == nullptr || triangles3 == nullptr ||
            output_status == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX scene build received a null buffer",
                        error_text, error_capacity);
        }
        if (vertex_count == 0 || triangle_count == 0 || vertex_count > UINT32_MAX ||
            triangle_count > UINT32_MAX || scene_signature == 0 || (rebuild != 0 && rebuild != 1)) {
            return fail(HS_STATUS_RANGE_ERROR, "OptiX scene dimensions or scalars are invalid",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (!rebuild && handle->tr_triangles != 0 && handle->tr_signature == scene_signature) {
            const cudaError_t e = cudaMemsetAsync(output_status, 0, sizeof(int32_t), nullptr);
            if (e != cudaSuccess) return cuda_failure(e, "write scene status", error_text, error_capacity);
            return ok(error_text, error_capacity);
        }
        cudaError_t e = hs::ensure_device_error(handle);
        if (e == cudaSuccess) e = cudaMemsetAsync(handle->device_error, 0, sizeof(uint32_t), nullptr);
        if (e != cudaSuccess) return cuda_failure(e, "trace scene build", error_text, error_capacity);
        if (handle->tr_pipeline_count == 0) handle->tr_pipeline_count = 1;
        bool bad_index = false;
        handle->tr_triangles = 0;
        handle->tr_signature = 0;
        e = hs::trace_build_scene(handle, vertices3, vertex_count, triangles3, triangle_count, &bad_index);
        if (bad_index) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "OptiX scene triangle names a vertex outside the vertex buffer", error_text,
                        error_capacity);
        }
        if (e != cudaSuccess) return cuda_failure(e, "trace scene build", error_text, error_capacity);
        handle->tr_signature = scene_signature;
        ++handle->tr_build_count;
        e = cudaMemsetAsync(output_status, 0, sizeof(int32_t), nullptr);
        if (e != cudaSuccess) return cuda_failure(e, "write scene status", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_optix_trace_f32_v1(
    HsRasterizerHandle handle, uint64_t ray_count, const float* ray_origins3,
    const float* ray_directions3, const float* background3, const float* means3d,
    const float* shs_m3, uint32_t coefficient_count, uint32_t degree, const float* others2,
    const float* opacities, const float* scales2, float scale_modifier, const float* rotations4,
    const float* viewmatrix4x4, const float* projmatrix4x4, const float* camera_position3,
    int32_t start_from_first, int32_t max_trace_depth, float specular_threshold, int32_t use_others,
    float* output_rgb3, float* output_depth1, float* output_acc1, float* output_normal3,
    float* output_dist1, float* output_aux2, float* output_mid32, float* output_wet1,
    char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX trace handle is null", error_text,
                        error_capacity);
        }
        if (ray_count > UINT32_MAX || coefficient_count == 0 || coefficient_count > 16 ||
            degree > 3 || coefficient_count < (degree + 1) * (degree + 1) ||
            (start_from_first != 0 && start_from_first != 1) || (use_others != 0 && use_others != 1) ||
            max_trace_depth < 0 || max_trace_depth > 1 || !std::isfinite(scale_modifier) ||
            scale_modifier <= 0.0f || !std::isfinite(specular_threshold)) {
            return fail(HS_STATUS_RANGE_ERROR, "OptiX trace dimensions or scalars are invalid",
                        error_text, error_capacity);
        }
        if (ray_count != 0 &&
            (ray_origins3 == nullptr || ray_directions3 == nullptr || background3 == nullptr ||
             means3d == nullptr || shs_m3 == nullptr || others2 == nullptr || opacities == nullptr ||
             scales2 == nullptr || rotations4 == nullptr || viewmatrix4x4 == nullptr ||
             projmatrix4x4 == nullptr || camera_position3 == nullptr || output_rgb3 == nullptr ||
             output_depth1 == nullptr || output_acc1 == nullptr || output_normal3 == nullptr ||
             output_dist1 == nullptr || output_aux2 == nullptr || output_mid32 == nullptr ||
             output_wet1 == nullptr)) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX trace received a null non-empty buffer",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->tr_triangles == 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX scene is not built", error_text,
                        error_capacity);
        }
        if (ray_count == 0) return ok(error_text, error_capacity);
        hs::TraceCall call;
        call.ray_count = ray_count;
        call.ray_origins3 = ray_origins3;
        call.ray_directions3 = ray_directions3;
        call.background3 = background3;
        call.means3d = means3d;
        call.shs_m3 = shs_m3;
        call.coefficient_count = coefficient_count;
        call.degree = degree;
        call.others2 = others2;
        call.opacities = opacities;
        call.scales2 = scales2;
        call.scale_modifier = scale_modifier;
        call.rotations4 = rotations4;
        call.viewmatrix4x4 = viewmatrix4x4;
        call.projmatrix4x4 = projmatrix4x4;
        call.camera_position3 = camera_position3;
        call.start_from_first = start_from_first;
        call.max_trace_depth = max_trace_depth;
        call.specular_threshold = specular_threshold;
        call.use_others = use_others;
        call.output_rgb3 = output_rgb3;
        call.output_depth1 = output_depth1;
        call.output_acc1 = output_acc1;
        call.output_normal3 = output_normal3;
        call.output_dist1 = output_dist1;
        call.output_aux2 = output_aux2;
        call.output_mid32 = output_mid32;
        call.output_wet1 = output_wet1;
        const cudaError_t e = hs::trace_rays(handle, call);
        if (e != cudaSuccess) return cuda_failure(e, "reflection trace", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_optix_workspace_stats_v1(HsRasterizerHandle handle, HsOptixWorkspaceStatsV1* stats,
                                    char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr || stats == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX stats received a null pointer", error_text,
                        error_capacity);
        }
        if (stats->struct_size != sizeof(HsOptixWorkspaceStatsV1) ||
            stats->abi_version != HS_RASTERIZER_ABI_VERSION) {
            return fail(HS_STATUS_ABI_MISMATCH, "OptiX stats ABI mismatch", error_text,
                        error_capacity);
        }
        std::lock_guard<std::mutex> lock(handle->mutex);
        stats->device = handle->device;
        stats->scene_ready = handle->tr_triangles != 0 ? 1u : 0u;
        stats->params_bytes = 0;
        stats->gas_output_bytes = handle->tr_scene.bytes;
        stats->gas_scratch_bytes = handle->tr_scratch.bytes;
        stats->dist3_bytes = 0;
        stats->current_bytes = hs::trace_current_bytes(handle);
        stats->peak_bytes = handle->tr_peak_bytes;
        stats->growth_count = handle->tr_growth_count;
        stats->scene_signature = handle->tr_signature;
        stats->gas_build_count = handle->tr_build_count;
        stats->pipeline_create_count = handle->tr_pipeline_count;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_optix_release_scene_v1(HsRasterizerHandle handle, char* error_text,
                                  uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX release handle is null", error_text,
                        error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        const cudaError_t e = hs::trace_release(handle);
        if (e != cudaSuccess) return cuda_failure(e, "release trace scene", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_precise_exp_f32_v1(const float* input, float* output, uint64_t count,
                                         char* error_text, uint64_t error_capacity) noexcept {
    return elementwise("precise_exp", count, input != nullptr && output != nullptr, error_text,
                       error_capacity, [&] { return hs::precise::exp(input, output, count, nullptr); });
}

int32_t hs_rasterizer_precise_sigmoid_f32_v1(const float* input, float* output, uint64_t count,
                                             char* error_text, uint64_t error_capacity) noexcept {
    return elementwise("precise_sigmoid", count, input != nullptr && output != nullptr, error_text,
                       error_capacity,
                       [&] { return hs::precise::sigmoid(input, output, count, nullptr); });
}

int32_t hs_rasterizer_precise_normalize4_f32_v1(const float* input4, float* output4,
                                                uint64_t count, char* error_text,
                                                uint64_t error_capacity) noexcept {
    return elementwise("precise_normalize4", count, input4 != nullptr && output4 != nullptr,
                       error_text, error_capacity,
                       [&] { return hs::precise::normalize4(input4, output4, count, nullptr); });
}

int32_t hs_rasterizer_precise_fuse_maps_f32_v1(const float* base_rgb, const float* reflection_rgb,
                                               const float* specular, float* diffuse,
                                               float* final_rgb, float* stored_reflection,
                                               uint64_t pixel_count, char* error_text,
                                               uint64_t error_capacity) noexcept {
    const bool present = base_rgb != nullptr && reflection_rgb != nullptr &&
                         specular != nullptr && diffuse != nullptr && final_rgb != nullptr &&
                         stored_reflection != nullptr;
    return elementwise("precise_fuse_maps", pixel_count, present, error_text, error_capacity, [&] {
        return hs::precise::fuse_maps(base_rgb, reflection_rgb, specular, diffuse, final_rgb,
                                      stored_reflection, pixel_count, nullptr);
    });
}

int32_t hs_rasterizer_precise_sh_to_rgb_f32_v1(const float* sh, const float* directions,
                                               uint64_t count, uint32_t coefficient_count,
                                               uint32_t degree, float* output, char* error_text,
                                               uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (degree > 3) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_sh_to_rgb supports degrees 0 through 3",
                        error_text, error_capacity);
        }
        if (coefficient_count < (degree + 1) * (degree + 1)) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_sh_to_rgb coefficient count is too small",
                        error_text, error_capacity);
        }
        if (count == 0) return ok(error_text, error_capacity);
        if (sh == nullptr || directions == nullptr || output == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "precise_sh_to_rgb received a null non-empty buffer",
                        error_text, error_capacity);
        }
        const cudaError_t e = hs::precise::sh_to_rgb(sh, directions, count, coefficient_count,
                                                     degree, output, nullptr);
        if (e != cudaSuccess) return cuda_failure(e, "precise_sh_to_rgb launch", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_precise_sh_colors5_f32_v1(const float* sh, uint32_t coefficient_count,
                                          uint32_t degree, const float* points,
                                          const float* center3, const float* specular,
                                          const float* roughness, uint64_t count,
                                          float* colors5, char* error_text,
                                          uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (degree > 3) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_sh_to_rgb supports degrees 0 through 3",
                        error_text, error_capacity);
        }
        if (coefficient_count < (degree + 1) * (degree + 1)) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_sh_to_rgb coefficient count is too small",
                        error_text, error_capacity);
        }
        if (count == 0) return ok(error_text, error_capacity);
        if (sh == nullptr || points == nullptr || center3 == nullptr || specular == nullptr ||
            roughness == nullptr || colors5 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "precise_sh_colors5 received a null non-empty buffer", error_text,
                        error_capacity);
        }
        const cudaError_t e = hs::precise::sh_colors5(sh, coefficient_count, degree, points,
                                                      center3, specular, roughness, count,
                                                      colors5, nullptr);
        if (e != cudaSuccess)
            return cuda_failure(e, "precise_sh_colors5 launch", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_precise_fuse_maps_planar_f32_v1(const float* base_rgb,
                                                const float* reflection_rgb,
                                                const float* specular, float* diffuse,
                                                float* final_rgb, float* stored_reflection,
                                                uint64_t pixel_count, char* error_text,
                                                uint64_t error_capacity) noexcept {
    const bool present = base_rgb != nullptr && reflection_rgb != nullptr &&
                         specular != nullptr && diffuse != nullptr && final_rgb != nullptr &&
                         stored_reflection != nullptr;
    return elementwise("precise_fuse_maps_planar", pixel_count, present, error_text,
                       error_capacity, [&] {
                           return hs::precise::fuse_maps_planar(base_rgb, reflection_rgb, specular,
                                                                diffuse, final_rgb,
                                                                stored_reflection, pixel_count,
                                                                nullptr);
                       });
}

int32_t hs_b200_pixel_rays_f32_v1(HsRasterizerHandle handle, int32_t width, int32_t height,
                                  const float* inverse_intrinsics3x3, const float* rotation3x3,
                                  float* scratch_n3, float* rays_n3, char* error_text,
                                  uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (width < 0 || height < 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "pixel_rays width and height must be non-negative",
                        error_text, error_capacity);
        }
        const uint64_t count = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
        if (count == 0) return ok(error_text, error_capacity);
        if (count > static_cast<uint64_t>(INT_MAX)) {
            return fail(HS_STATUS_RANGE_ERROR, "pixel_rays pixel count exceeds cuBLAS int range",
                        error_text, error_capacity);
        }
        if (handle == nullptr || inverse_intrinsics3x3 == nullptr || rotation3x3 == nullptr ||
            scratch_n3 == nullptr || rays_n3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "pixel_rays received a null buffer", error_text,
                        error_capacity);
        }
        if (scratch_n3 == rays_n3) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "pixel_rays scratch must not alias the rays",
                        error_text, error_capacity);
        }
        const cudaError_t prior = cudaGetLastError();
        if (prior != cudaSuccess)
            return cuda_failure(prior, "pixel_rays preexisting CUDA error", error_text, error_capacity);
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->math_tf32_blas == nullptr) {
            return fail(HS_STATUS_INTERNAL_ERROR, "pixel_rays math context is not initialized",
                        error_text, error_capacity);
        }
        // depth_to_normal (math.py:360-401): pixels (x, y, 1), then
        // camera rays = pixels @ K^-T and world rays = camera rays @ R^T, each
        // the TF32 GEMM of precise_matmul_nt_n3k3: one tensor-core kernel
        // (postprocess.cu), or for images of fewer than kMmaMinRows pixels the
        // cuBLAS calls themselves through the scratch buffer.
        if (count >= hs::post::kMmaMinRows) {
            const cudaError_t ce = hs::post::pixel_rays(width, height, inverse_intrinsics3x3,
                                                        rotation3x3, rays_n3, nullptr);
            if (ce != cudaSuccess) return cuda_failure(ce, "pixel_rays execution", error_text, error_capacity);
        } else {
            cudaError_t ce = hs::post::pixel_grid(width, height, rays_n3, nullptr);
            if (ce != cudaSuccess) return cuda_failure(ce, "pixel_rays grid", error_text, error_capacity);
            const float alpha = 1.0f, beta = 0.0f;
            cublasStatus_t bs = cublasSgemm(handle->math_tf32_blas, CUBLAS_OP_T, CUBLAS_OP_N, 3,
                                            static_cast<int>(count), 3, &alpha, inverse_intrinsics3x3, 3,
                                            rays_n3, 3, &beta, scratch_n3, 3);
            if (bs == CUBLAS_STATUS_SUCCESS) {
                bs = cublasSgemm(handle->math_tf32_blas, CUBLAS_OP_T, CUBLAS_OP_N, 3,
                                 static_cast<int>(count), 3, &alpha, rotation3x3, 3, scratch_n3, 3,
                                 &beta, rays_n3, 3);
            }
            if (bs != CUBLAS_STATUS_SUCCESS)
                return cublas_failure(bs, "pixel_rays cublasSgemm", error_text, error_capacity);
            ce = cudaGetLastError();
            if (ce != cudaSuccess) return cuda_failure(ce, "pixel_rays execution", error_text, error_capacity);
        }
        handle->math_matmul_calls += 2;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_standard_postprocess_f32_v1(
    int32_t width, int32_t height, const float* color5, const float* aux7, const float* rays_n3,
    const float* origin3, const float* normal_rotation3x3, double depth_ratio, float* rgb_map3,
    float* acc_map, float* dpt_map, float* norm_map3, float* surf_norm_map3, float* dist_map,
    float* spec_map, float* rough_map, char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (width < 0 || height < 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "standard_postprocess width and height must be non-negative", error_text,
                        error_capacity);
        }
        if (!std::isfinite(depth_ratio)) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "standard_postprocess depth_ratio must be finite", error_text,
                        error_capacity);
        }
        const uint64_t pixels = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
        const bool present = color5 != nullptr && aux7 != nullptr && rays_n3 != nullptr &&
                             origin3 != nullptr && normal_rotation3x3 != nullptr &&
                             rgb_map3 != nullptr && acc_map != nullptr && dpt_map != nullptr &&
                             norm_map3 != nullptr && surf_norm_map3 != nullptr &&
                             dist_map != nullptr && spec_map != nullptr && rough_map != nullptr;
        // (1 - ratio) and ratio as float32 scalars of a double ratio (math.py:440-442).
        const float keep = static_cast<float>(1.0 - depth_ratio);
        const float ratio = static_cast<float>(depth_ratio);
        return elementwise("standard_postprocess", pixels, present, error_text, error_capacity, [&] {
            const hs::post::StandardMaps maps{rgb_map3,       acc_map,  dpt_map,  norm_map3,
                                              surf_norm_map3, dist_map, spec_map, rough_map};
            return hs::post::standard(width, height, color5, aux7, rays_n3, origin3,
                                      normal_rotation3x3, keep, ratio, maps, nullptr);
        });
    });
}

int32_t hs_b200_flashgs_postprocess_f32_v1(int32_t width, int32_t height, const float* color3,
                                           const float* other2, const float* depth1,
                                           const float* alpha1, const float* normal3,
                                           const float* normal_rotation3x3, float* rgb_map3,
                                           float* acc_map, float* dpt_map, float* norm_map3,
                                           float* surf_norm_map3, float* dist_map,
                                           float* spec_map, char* error_text,
                                           uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (width < 0 || height < 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "flashgs_postprocess width and height must be non-negative", error_text,
                        error_capacity);
        }
        const uint64_t pixels = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
        const bool present = color3 != nullptr && other2 != nullptr && depth1 != nullptr &&
                             alpha1 != nullptr && normal3 != nullptr &&
                             normal_rotation3x3 != nullptr && rgb_map3 != nullptr &&
                             acc_map != nullptr && dpt_map != nullptr && norm_map3 != nullptr &&
                             spec_map != nullptr;
        return elementwise("flashgs_postprocess", pixels, present, error_text, error_capacity, [&] {
            const hs::post::FlashgsMaps maps{rgb_map3, acc_map,  dpt_map, norm_map3,
                                             surf_norm_map3, dist_map, spec_map};
            return hs::post::flashgs(width, height, color3, other2, depth1, alpha1, normal3,
                                     normal_rotation3x3, maps, nullptr);
        });
    });
}

int32_t hs_rasterizer_precise_direction_f32_v1(const float* points, const float* center,
                                               uint64_t count, float* output, char* error_text,
                                               uint64_t error_capacity) noexcept {
    return elementwise("precise_direction", count,
                       points != nullptr && center != nullptr && output != nullptr, error_text,
                       error_capacity,
                       [&] { return hs::precise::direction(points, center, count, output, nullptr); });
}

int32_t hs_rasterizer_precise_camera_center_f32_v2(HsRasterizerHandle handle,
                                                   const float* rotation3x3,
                                                   const float* translation3x1, float* output3,
                                                   char* error_text,
                                                   uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr || rotation3x3 == nullptr || translation3x1 == nullptr ||
            output3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "precise_camera_center received a null buffer",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->math_workspace == nullptr || handle->math_tf32_blas == nullptr) {
            return fail(HS_STATUS_INTERNAL_ERROR, "precise_camera_center math context is not initialized",
                        error_text, error_capacity);
        }
        float* negative = reinterpret_cast<float*>(math_at(handle, kMathCameraOffset));
        const cudaError_t ce = hs::precise::negate9(rotation3x3, negative, nullptr);
        if (ce != cudaSuccess)
            return cuda_failure(ce, "precise_camera_center negative-R", error_text, error_capacity);
        // output[1x3] = t[1x3] * (-R)^T as in reference c_api.cpp:1390-1407.
        const float alpha = 1.0f, beta = 0.0f;
        const cublasStatus_t bs = cublasSgemm(handle->math_tf32_blas, CUBLAS_OP_N, CUBLAS_OP_T, 1,
                                              3, 3, &alpha, translation3x1, 1, negative, 3, &beta,
                                              output3, 1);
        if (bs != CUBLAS_STATUS_SUCCESS)
            return cublas_failure(bs, "precise_camera_center SGEMM", error_text, error_capacity);
        ++handle->math_camera_center_calls;
        return ok(error_text, error_capacity);
    });
}

namespace {

// Buffers of one general inverse (device memory of the math workspace).
struct InverseBuffers {
    float* factor;
    float* rhs;
    float* work;
    int* pivots;
    int* info;
    float** factor_array;  // device array holding `factor`
    float** rhs_array;     // device array holding `rhs`
};

InverseBuffers inverse_buffers(HsRasterizerContext* c, uint64_t base) {
    return InverseBuffers{reinterpret_cast<float*>(math_at(c, base + kMathFactorOffset)),
                          reinterpret_cast<float*>(math_at(c, base + kMathRhsOffset)),
                          reinterpret_cast<float*>(math_at(c, base + kMathSolverWorkspaceOffset)),
                          reinterpret_cast<int*>(math_at(c, base + kMathPivotsOffset)),
                          reinterpret_cast<int*>(math_at(c, base + kMathInfoOffset)),
                          reinterpret_cast<float**>(math_at(c, base + kMathFactorArrayOffset)),
                          reinterpret_cast<float**>(math_at(c, base + kMathRhsArrayOffset))};
}

// linalg_inv_ex as in reference c_api.cpp:1493-1600: identity RHS, LU of the
// row-major n x n `input` read as column-major A^T (cusolverDnSgetrf), getrs
// with OP_T (cublasSgetrsBatched), the column-major solution transposed into
// row-major `output`. The caller holds the handle's mutex and has bound the
// handle's solver and TF32 BLAS to `stream`.
int32_t general_inverse(HsRasterizerContext* h, const float* input, int n, const InverseBuffers& b,
                        float* output, cudaStream_t stream, char* error_text, uint64_t error_capacity) {
    const size_t bytes = static_cast<size_t>(n) * n * sizeof(float);
    cudaError_t ce = cudaMemcpyAsync(b.rhs, math_at(h, n == 3 ? kMathIdentity3Offset : kMathIdentity4Offset),
                                     bytes, cudaMemcpyDeviceToDevice, stream);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(b.factor, input, bytes, cudaMemcpyDeviceToDevice, stream);
    if (ce != cudaSuccess)
        return cuda_failure(ce, "precise_general_inverse identity/input copy", error_text, error_capacity);
    int work_count = 0;
    cusolverStatus_t ss = cusolverDnSgetrf_bufferSize(h->math_solver, n, n, b.factor, n, &work_count);
    if (ss != CUSOLVER_STATUS_SUCCESS)
        return cusolver_failure(ss, "precise_general_inverse cusolverDnSgetrf_bufferSize", error_text,
                                error_capacity);
    if (work_count > h->math_inverse_workspace_count) {
        return fail(HS_STATUS_RANGE_ERROR, "precise_general_inverse persistent workspace is too small",
                    error_text, error_capacity);
    }
    ss = cusolverDnSgetrf(h->math_solver, n, n, b.factor, n, b.work, b.pivots, b.info);
    if (ss != CUSOLVER_STATUS_SUCCESS)
        return cusolver_failure(ss, "precise_general_inverse cusolverDnSgetrf", error_text, error_capacity);
    int32_t* solve_info = &h->math_solve_info[h->math_general_inverse_calls % 16];
    *solve_info = 0;
    const cublasStatus_t bs = cublasSgetrsBatched(h->math_tf32_blas, CUBLAS_OP_T, n, n, b.factor_array, n,
                                                  b.pivots, b.rhs_array, n, solve_info, 1);
    if (bs != CUBLAS_STATUS_SUCCESS)
        return cublas_failure(bs, "precise_general_inverse cublasSgetrsBatched", error_text, error_capacity);
    ce = hs::precise::column_to_row_major(b.rhs, static_cast<uint32_t>(n), output, stream);
    if (ce != cudaSuccess)
        return cuda_failure(ce, "precise_general_inverse output transpose", error_text, error_capacity);
    ++h->math_general_inverse_calls;
    return HS_STATUS_OK;
}

}  // namespace

int32_t hs_rasterizer_precise_general_inverse_f32_v2(HsRasterizerHandle handle,
                                                     const float* input, uint32_t dimension,
                                                     float* output, char* error_text,
                                                     uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (dimension != 3 && dimension != 4) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_general_inverse dimension must be 3 or 4",
                        error_text, error_capacity);
        }
        if (handle == nullptr || input == nullptr || output == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "precise_general_inverse received a null buffer",
                        error_text, error_capacity);
        }
        const cudaError_t prior = cudaGetLastError();
        if (prior != cudaSuccess) {
            return cuda_failure(prior, "precise_general_inverse preexisting CUDA error", error_text,
                                error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->math_workspace == nullptr || handle->math_solver == nullptr ||
            handle->math_tf32_blas == nullptr) {
            return fail(HS_STATUS_INTERNAL_ERROR,
                        "precise_general_inverse math context is not initialized", error_text,
                        error_capacity);
        }
        const int32_t status = general_inverse(handle, input, static_cast<int>(dimension),
                                               inverse_buffers(handle, 0), output, nullptr, error_text,
                                               error_capacity);
        if (status != HS_STATUS_OK) return status;
        const cudaError_t trailing = cudaGetLastError();
        if (trailing != cudaSuccess)
            return cuda_failure(trailing, "precise_general_inverse trailing CUDA error", error_text,
                                error_capacity);
        return ok(error_text, error_capacity);
    });
}

namespace {

// The view's camera terms of the standard postprocess on `stream`
// (hs_b200_postprocess_camera_f32_v1 after its argument checks; the caller
// holds h's mutex on h's device).
// captured: queued inside a stream capture, whose caller orders the graph's
// launches after view_camera_event and records it after them (an event
// recorded outside a capture cannot be waited on inside it).
int32_t camera_terms(HsRasterizerContext* h, int32_t width, int32_t height, double fov_x, double fov_y,
                     const float* world_view4x4, float* camera30, float* rays_n3, cudaStream_t stream,
                     char* error_text, uint64_t error_capacity, bool captured = false) {
    const uint64_t count = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
    // The intrinsics as depth_to_normal builds them (math.py:338-389):
    // focal = float32(length) / float32(2 tan(float32(fov) / 2)) with the
    // tangent in double, principal point float32(length) / 2.
    auto focal = [](int length, double fov) {
        const float half = static_cast<float>(fov) / 2.0f;
        const float denominator = static_cast<float>(2.0 * std::tan(static_cast<double>(half)));
        return static_cast<float>(length) / denominator;
    };
    const float fx = focal(width, fov_x), fy = focal(height, fov_y);
    const float cx = static_cast<float>(width) / 2.0f, cy = static_cast<float>(height) / 2.0f;
    const cudaStream_t s = stream;
    float* k9 = reinterpret_cast<float*>(math_at(h, kMathViewK));
    float* wt16 = reinterpret_cast<float*>(math_at(h, kMathViewWt));
    float* c2w16 = reinterpret_cast<float*>(math_at(h, kMathViewC2w));
    // the region is this entry's own: order after the previous call's use of it
    cudaError_t ce = cudaSuccess;
    if (h->view_camera_event == nullptr) {
        ce = cudaEventCreateWithFlags(&h->view_camera_event, cudaEventDisableTiming);
    } else if (!captured) {
        ce = cudaStreamWaitEvent(s, h->view_camera_event, 0);
    }
    if (ce == cudaSuccess) ce = hs::post::camera_inputs(fx, cx, fy, cy, world_view4x4, k9, wt16, s);
    if (ce != cudaSuccess) return cuda_failure(ce, "postprocess_camera inputs", error_text, error_capacity);
    // the two inverses of precise_general_inverse, on `stream`
    cublasStatus_t bs = cublasSetStream(h->math_tf32_blas, s);
    cusolverStatus_t ss = cusolverDnSetStream(h->math_solver, s);
    int32_t status = HS_STATUS_OK;
    if (bs != CUBLAS_STATUS_SUCCESS) {
        status = cublas_failure(bs, "postprocess_camera cublasSetStream", error_text, error_capacity);
    } else if (ss != CUSOLVER_STATUS_SUCCESS) {
        status = cusolver_failure(ss, "postprocess_camera cusolverDnSetStream", error_text, error_capacity);
    } else {
        const InverseBuffers view = inverse_buffers(h, kMathViewOffset);
        status = general_inverse(h, k9, 3, view, camera30, s, error_text, error_capacity);
        if (status == HS_STATUS_OK)
            status = general_inverse(h, wt16, 4, view, c2w16, s, error_text, error_capacity);
        // images under kMmaMinRows pixels: the reference's cuBLAS products on this stream
        if (status == HS_STATUS_OK && count < hs::post::kMmaMinRows) {
            float* scratch = reinterpret_cast<float*>(math_at(h, kMathViewRays));
            ce = hs::post::camera_pack(c2w16, world_view4x4, camera30, s);
            if (ce == cudaSuccess) ce = hs::post::pixel_grid(width, height, rays_n3, s);
            const float alpha = 1.0f, beta = 0.0f;
            if (ce != cudaSuccess) {
                status = cuda_failure(ce, "postprocess_camera rays", error_text, error_capacity);
            } else {
                bs = cublasSgemm(h->math_tf32_blas, CUBLAS_OP_T, CUBLAS_OP_N, 3, static_cast<int>(count),
                                 3, &alpha, camera30, 3, rays_n3, 3, &beta, scratch, 3);
                if (bs == CUBLAS_STATUS_SUCCESS)
                    bs = cublasSgemm(h->math_tf32_blas, CUBLAS_OP_T, CUBLAS_OP_N, 3, static_cast<int>(count),
                                     3, &alpha, camera30 + 9, 3, scratch, 3, &beta, rays_n3, 3);
                if (bs != CUBLAS_STATUS_SUCCESS)
                    status = cublas_failure(bs, "postprocess_camera cublasSgemm", error_text, error_capacity);
            }
        }
    }
    // the handles go back to the legacy default stream of the other helpers
    const cublasStatus_t rb = cublasSetStream(h->math_tf32_blas, nullptr);
    const cusolverStatus_t rs = cusolverDnSetStream(h->math_solver, nullptr);
    if (status != HS_STATUS_OK) return status;
    if (rb != CUBLAS_STATUS_SUCCESS)
        return cublas_failure(rb, "postprocess_camera cublasSetStream", error_text, error_capacity);
    if (rs != CUSOLVER_STATUS_SUCCESS)
        return cusolver_failure(rs, "postprocess_camera cusolverDnSetStream", error_text, error_capacity);
    if (count >= hs::post::kMmaMinRows) {
        ce = hs::post::camera_pack(c2w16, world_view4x4, camera30, s);
        if (ce == cudaSuccess) ce = hs::post::pixel_rays(width, height, camera30, camera30 + 9, rays_n3, s);
        if (ce != cudaSuccess) return cuda_failure(ce, "postprocess_camera rays", error_text, error_capacity);
    }
    if (!captured) {
        ce = cudaEventRecord(h->view_camera_event, s);
        if (ce != cudaSuccess) return cuda_failure(ce, "postprocess_camera event", error_text, error_capacity);
    }
    h->math_matmul_calls += 2;
    return HS_STATUS_OK;
}

}  // namespace

int32_t hs_b200_postprocess_camera_f32_v1(HsRasterizerHandle handle, int32_t width, int32_t height,
                                          double fov_x, double fov_y, const float* world_view4x4,
                                          float* camera30, float* rays_n3, void* stream, char* error_text,
                                          uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (width <= 0 || height <= 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "postprocess_camera width and height must be positive",
                        error_text, error_capacity);
        }
        const uint64_t count = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
        if (count > static_cast<uint64_t>(INT_MAX)) {
            return fail(HS_STATUS_RANGE_ERROR, "postprocess_camera pixel count exceeds cuBLAS int range",
                        error_text, error_capacity);
        }
        if (!std::isfinite(fov_x) || !std::isfinite(fov_y)) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "postprocess_camera fields of view must be finite",
                        error_text, error_capacity);
        }
        if (handle == nullptr || world_view4x4 == nullptr || camera30 == nullptr || rays_n3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "postprocess_camera received a null buffer", error_text,
                        error_capacity);
        }
        const cudaError_t prior = cudaGetLastError();
        if (prior != cudaSuccess)
            return cuda_failure(prior, "postprocess_camera preexisting CUDA error", error_text, error_capacity);
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->math_workspace == nullptr || handle->math_solver == nullptr ||
            handle->math_tf32_blas == nullptr) {
            return fail(HS_STATUS_INTERNAL_ERROR, "postprocess_camera math context is not initialized",
                        error_text, error_capacity);
        }
        const int32_t status = camera_terms(handle, width, height, fov_x, fov_y, world_view4x4, camera30, rays_n3,
                                            static_cast<cudaStream_t>(stream), error_text, error_capacity);
        if (status != HS_STATUS_OK) return status;
        handle->math_matmul_calls += 2;
        const cudaError_t trailing = cudaGetLastError();
        if (trailing != cudaSuccess)
            return cuda_failure(trailing, "postprocess_camera execution", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_precise_matmul_nt_n3k3_f32_v2(HsRasterizerHandle handle,
                                                    const float* left_n3, const float* right3x3,
                                                    uint64_t count, float* output_n3,
                                                    char* error_text,
                                                    uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (count == 0) return ok(error_text, error_capacity);
        if (count > static_cast<uint64_t>(INT_MAX)) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_matmul_nt_n3k3 count exceeds cuBLAS int range",
                        error_text, error_capacity);
        }
        if (handle == nullptr || left_n3 == nullptr || right3x3 == nullptr || output_n3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "precise_matmul_nt_n3k3 received a null non-empty buffer", error_text,
                        error_capacity);
        }
        const cudaError_t prior = cudaGetLastError();
        if (prior != cudaSuccess) {
            return cuda_failure(prior, "precise_matmul_nt_n3k3 preexisting CUDA error", error_text,
                                error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->math_tf32_blas == nullptr) {
            return fail(HS_STATUS_INTERNAL_ERROR, "precise_matmul_nt_n3k3 math context is not initialized",
                        error_text, error_capacity);
        }
        // cublasSgemm(OP_T, OP_N, 3, count, 3) under TF32 tensor-op math in the
        // reference; the same MMA products here (postprocess.cu), and that
        // call itself below kMmaMinRows rows, where cuBLAS takes another path.
        if (count >= hs::post::kMmaMinRows) {
            const cudaError_t e = hs::post::matmul_nt_n3k3(left_n3, right3x3, count, output_n3, nullptr);
            if (e != cudaSuccess)
                return cuda_failure(e, "precise_matmul_nt_n3k3 execution", error_text, error_capacity);
        } else {
            const float alpha = 1.0f, beta = 0.0f;
            const cublasStatus_t bs = cublasSgemm(handle->math_tf32_blas, CUBLAS_OP_T, CUBLAS_OP_N, 3,
                                                  static_cast<int>(count), 3, &alpha, right3x3, 3,
                                                  left_n3, 3, &beta, output_n3, 3);
            if (bs != CUBLAS_STATUS_SUCCESS)
                return cublas_failure(bs, "precise_matmul_nt_n3k3 cublasSgemm", error_text, error_capacity);
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess)
                return cuda_failure(e, "precise_matmul_nt_n3k3 execution", error_text, error_capacity);
        }
        ++handle->math_matmul_calls;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_precise_pixel_world_f32_v2(HsRasterizerHandle handle,
                                                 const float* rotation3x3,
                                                 const float* vectors_n3, uint64_t count,
                                                 float* output_n3, char* error_text,
                                                 uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (count == 0) return ok(error_text, error_capacity);
        if (count > static_cast<uint64_t>(INT_MAX)) {
            return fail(HS_STATUS_RANGE_ERROR, "precise_pixel_world count exceeds cuBLAS int range",
                        error_text, error_capacity);
        }
        if (handle == nullptr || rotation3x3 == nullptr || vectors_n3 == nullptr ||
            output_n3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "precise_pixel_world received a null non-empty buffer",
                        error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        if (handle->math_default_blas == nullptr) {
            return fail(HS_STATUS_INTERNAL_ERROR, "precise_pixel_world math context is not initialized",
                        error_text, error_capacity);
        }
        const float alpha = 1.0f, beta = 0.0f;
        const cublasStatus_t bs = cublasGemmStridedBatchedEx(
            handle->math_default_blas, CUBLAS_OP_N, CUBLAS_OP_N, 3, 1, 3, &alpha, rotation3x3,
            CUDA_R_32F, 3, 0, vectors_n3, CUDA_R_32F, 3, 3, &beta, output_n3, CUDA_R_32F, 3, 3,
            static_cast<int>(count), CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        if (bs != CUBLAS_STATUS_SUCCESS)
            return cublas_failure(bs, "precise_pixel_world batched GEMM", error_text, error_capacity);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_failure(e, "precise_pixel_world execution", error_text, error_capacity);
        ++handle->math_pixel_world_calls;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_rasterizer_precise_disk_rotation_f32_v1(const float* rotation_wxyz, uint64_t count,
                                                   float* rotation_matrix9, char* error_text,
                                                   uint64_t error_capacity) noexcept {
    return elementwise("precise_disk_rotation", count,
                       rotation_wxyz != nullptr && rotation_matrix9 != nullptr, error_text,
                       error_capacity, [&] {
                           return hs::precise::disk_rotation(rotation_wxyz, count, rotation_matrix9,
                                                             nullptr);
                       });
}

int32_t hs_rasterizer_precise_reflection_prefix_f32_v1(const float* rotation_wxyz,
                                                       uint64_t count, float* rotation_matrix9,
                                                       char* error_text,
                                                       uint64_t error_capacity) noexcept {
    return elementwise("precise_reflection_prefix", count,
                       rotation_wxyz != nullptr && rotation_matrix9 != nullptr, error_text,
                       error_capacity, [&] {
                           return hs::precise::reflection_prefix(rotation_wxyz, count,
                                                                 rotation_matrix9, nullptr);
                       });
}

int32_t hs_rasterizer_precise_reflection_suffix_f32_v1(const float* xyz,
                                                       const float* camera_center,
                                                       const float* normal_raw3, uint64_t count,
                                                       float* output36, char* error_text,
                                                       uint64_t error_capacity) noexcept {
    return elementwise("precise_reflection_suffix", count,
                       xyz != nullptr && camera_center != nullptr && normal_raw3 != nullptr &&
                           output36 != nullptr,
                       error_text, error_capacity, [&] {
                           return hs::precise::reflection_suffix(xyz, camera_center, normal_raw3,
                                                                 count, output36, nullptr);
                       });
}

// ---- extensions of this library (no counterpart in the reference ABI) ----

int32_t hs_b200_test_stall_lookback_v1(HsRasterizerHandle handle, uint32_t tile,
                                       char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (handle == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "handle is null", error_text, error_capacity);
        }
        std::lock_guard<std::mutex> lock(handle->mutex);
        handle->test_stall_tile = tile;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_stage_timing_enable_v1(HsRasterizerHandle handle, int32_t enable, char* error_text,
                                       uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        handle->timer.enabled = enable != 0;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_stage_timing_read_v1(HsRasterizerHandle handle, double* stage_ms3,
                                     uint64_t* raster_calls, char* error_text,
                                     uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (stage_ms3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "stage_ms3 is null", error_text, error_capacity);
        }
        const int32_t ds = select_device(handle, error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        std::lock_guard<std::mutex> lock(handle->mutex);
        const cudaError_t e = hs::stage_timing_read(handle->timer, stage_ms3, raster_calls);
        if (e != cudaSuccess) return cuda_failure(e, "stage timing", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_rasterizer_forward_noalloc_f32_v1(
    int32_t device, uint64_t point_count, const float* background5, int32_t width,
    int32_t height, const float* means3d, const float* colors5, const float* opacities,
    const float* scales2, float scale_modifier, const float* rotations4,
    const float* viewmatrix4x4, const float* projmatrix4x4, const float* camera_position3,
    float tan_fovx, float tan_fovy, int32_t prefiltered, float* output_color5, float* output_aux7,
    float* output_weight, int32_t* output_radii, int32_t* output_rendered, char* error_text,
    uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        // Same argument checks as hs_rasterizer_forward_f32_v1, with a device
        // ordinal in place of the context handle.
        if (background5 == nullptr || output_color5 == nullptr || output_aux7 == nullptr ||
            output_rendered == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "rasterizer received a null required handle or buffer", error_text,
                        error_capacity);
        }
        if (point_count > static_cast<uint64_t>(INT_MAX) || width <= 0 || height <= 0 ||
            !std::isfinite(scale_modifier) || !std::isfinite(tan_fovx) ||
            !std::isfinite(tan_fovy) || tan_fovx <= 0.0f || tan_fovy <= 0.0f ||
            (prefiltered != 0 && prefiltered != 1)) {
            return fail(HS_STATUS_RANGE_ERROR, "rasterizer dimensions or scalar arguments are invalid",
                        error_text, error_capacity);
        }
        if (point_count != 0 &&
            (means3d == nullptr || colors5 == nullptr || opacities == nullptr ||
             scales2 == nullptr || rotations4 == nullptr || viewmatrix4x4 == nullptr ||
             projmatrix4x4 == nullptr || camera_position3 == nullptr ||
             output_weight == nullptr || output_radii == nullptr)) {
            return fail(HS_STATUS_INVALID_ARGUMENT,
                        "non-empty rasterizer input contains a null buffer", error_text,
                        error_capacity);
        }
        int device_count = 0;
        cudaError_t e = cudaGetDeviceCount(&device_count);
        if (e != cudaSuccess) return cuda_failure(e, "cudaGetDeviceCount", error_text, error_capacity);
        if (device < 0 || device >= device_count) {
            return fail(HS_STATUS_RANGE_ERROR, "device is outside the visible CUDA device range",
                        error_text, error_capacity);
        }
        DeviceGuard device_guard;
        e = device_guard.select(device);
        if (e != cudaSuccess) return cuda_failure(e, "cudaSetDevice", error_text, error_capacity);
        char limit[256] = {};
        e = hs::standard_forward_noalloc(
            device, static_cast<int32_t>(point_count), background5, width, height, means3d,
            colors5, opacities, scales2, scale_modifier, rotations4, viewmatrix4x4,
            projmatrix4x4, prefiltered != 0, output_color5, output_aux7, output_weight,
            output_radii, output_rendered, limit, sizeof(limit));
        if (limit[0] != '\0') return fail(HS_STATUS_RANGE_ERROR, limit, error_text, error_capacity);
        if (e != cudaSuccess) {
            return cuda_failure(e, "no-alloc five-channel rasterizer forward", error_text,
                                error_capacity);
        }
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_flashgs_forward_rows_f32_v1(
    HsRasterizerHandle handle, uint32_t tile_row_begin, uint32_t tile_row_end,
    uint64_t point_count, int32_t width, int32_t height, const float* positions3,
    const float* shs48, const float* colors3, int32_t use_sh, const float* opacities1,
    const float* covariance6, const float* scales2, float scale_modifier, const float* rotations4,
    const float* specular1, const float* roughness1, const float* camera_position3,
    const float* camera_rotation9, float focal_x, float focal_y, float z_far, float z_near,
    const float* background3, uint64_t initial_pair_capacity, float* output_color3,
    float* output_other2, float* output_depth1, float* output_alpha1, float* output_normal3,
    float* output_median_depth1, float* output_distortion1, int32_t* output_num_rendered,
    char* error_text, uint64_t error_capacity) noexcept {
    HsB200FlashgsCallV2 a = flashgs_args(
        handle, point_count, width, height, positions3, shs48, colors3, use_sh, opacities1,
        covariance6, scales2, scale_modifier, rotations4, specular1, roughness1, camera_position3,
        camera_rotation9, focal_x, focal_y, z_far, z_near, background3, initial_pair_capacity,
        output_color3, output_other2, output_depth1, output_alpha1, output_normal3,
        output_median_depth1, output_distortion1, output_num_rendered);
    a.tile_row_begin = tile_row_begin;
    // an explicit strip: UINT32_MAX is out of range here, not "whole frame"
    a.tile_row_end = tile_row_end == UINT32_MAX ? UINT32_MAX - 1 : tile_row_end;
    return flashgs_entry(a, error_text, error_capacity);
}

int32_t hs_b200_rasterizer_forward_rows_f32_v1(
    HsRasterizerHandle handle, uint32_t tile_row_begin, uint32_t tile_row_end,
    uint64_t point_count, const float* background5, int32_t width, int32_t height,
    const float* means3d, const float* colors5, const float* opacities, const float* scales2,
    float scale_modifier, const float* rotations4, const float* viewmatrix4x4,
    const float* projmatrix4x4, const float* camera_position3, float tan_fovx, float tan_fovy,
    int32_t prefiltered, float* output_color5, float* output_aux7, float* output_weight,
    int32_t* output_radii, int32_t* output_rendered, char* error_text,
    uint64_t error_capacity) noexcept {
    HsB200RasterizerCallV2 a = rasterizer_args(
        handle, point_count, background5, width, height, means3d, colors5, opacities, scales2,
        scale_modifier, rotations4, viewmatrix4x4, projmatrix4x4, camera_position3, tan_fovx,
        tan_fovy, prefiltered, output_color5, output_aux7, output_weight, output_radii,
        output_rendered);
    a.tile_row_begin = tile_row_begin;
    a.tile_row_end = tile_row_end == UINT32_MAX ? UINT32_MAX - 1 : tile_row_end;
    return rasterizer_entry(a, error_text, error_capacity);
}

int32_t hs_b200_standard_view_v2(const HsB200StandardViewV2* v, char* error_text,
                                 uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (v == nullptr || v->struct_size < sizeof(HsB200StandardViewV2)) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "standard view is null or its struct_size is too small",
                        error_text, error_capacity);
        }
        // the two raster calls, checked as the concurrent entry checks them
        auto raster_args = [&](const HsB200StandardGroupV2& g, HsRasterizerHandle handle) {
            HsB200RasterizerCallV2 a{};
            a.handle = handle;
            a.point_count = g.count;
            a.background5 = g.background5;
            a.width = v->width;
            a.height = v->height;
            a.means3d = g.means3d;
            a.colors5 = g.colors5;
            a.opacities = g.opacities;
            a.scales2 = g.scales2;
            a.scale_modifier = 1.0f;
            a.prefiltered = 0;
            a.rotations4 = g.rotations4;
            a.viewmatrix4x4 = v->viewmatrix4x4;
            a.projmatrix4x4 = v->projmatrix4x4;
            a.camera_position3 = v->camera_position3;
            a.tan_fovx = v->tan_fovx;
            a.tan_fovy = v->tan_fovy;
            a.output_color5 = g.output_color5;
            a.output_aux7 = g.output_aux7;
            a.output_weight = g.output_weight;
            a.output_radii = g.output_radii;
            a.output_rendered = g.output_rendered;
            a.tile_row_begin = 0;
            a.tile_row_end = UINT32_MAX;
            return a;
        };
        hs::StandardCall calls[2];
        HsRasterizerContext* contexts[2] = {v->base_handle, v->reflection_handle};
        const HsB200RasterizerCallV2 base_args = raster_args(v->base, v->base_handle);
        const HsB200RasterizerCallV2 refl_args = raster_args(v->reflection, v->reflection_handle);
        int32_t cs = check_rasterizer(base_args, &calls[0], error_text, error_capacity);
        if (cs == HS_STATUS_OK) cs = check_rasterizer(refl_args, &calls[1], error_text, error_capacity);
        if (cs != HS_STATUS_OK) return cs;
        if (contexts[0] == contexts[1]) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "standard view needs two distinct handles", error_text,
                        error_capacity);
        }
        const uint64_t nb = v->base.count, nr = v->reflection.count;
        if (v->sh_coefficients == 0 || v->sh_coefficients > 16 || v->sh_degree > 3 ||
            v->sh_coefficients < (v->sh_degree + 1) * (v->sh_degree + 1)) {
            return fail(HS_STATUS_RANGE_ERROR, "standard view SH dimensions are invalid", error_text,
                        error_capacity);
        }
        if ((nb != 0 && (v->base_sh == nullptr || v->base.specular == nullptr || v->base.roughness == nullptr)) ||
            (nr != 0 && (v->reflection_rotation_raw4 == nullptr || v->reflection_rotation9 == nullptr ||
                         v->reflection_normal3 == nullptr || v->reflection_rays36 == nullptr ||
                         v->reflection.specular == nullptr || v->reflection.roughness == nullptr ||
                         (v->trace == 0 && v->reflection_rgb3 == nullptr))) ||
            v->fused_rgb3 == nullptr || v->diffuse_rgb3 == nullptr || v->reflection_rgb_map3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "standard view received a null required buffer", error_text,
                        error_capacity);
        }
        const int32_t ts = check_view_trace(*v, nr, v->reflection_shs, v->reflection_others2, "standard view",
                                            error_text, error_capacity);
        if (ts != HS_STATUS_OK) return ts;
        const bool post = v->camera30 != nullptr;
        const uint64_t pixels = static_cast<uint64_t>(v->width) * static_cast<uint64_t>(v->height);
        if (post) {
            if (!std::isfinite(v->fov_x) || !std::isfinite(v->fov_y) || !std::isfinite(v->depth_ratio)) {
                return fail(HS_STATUS_INVALID_ARGUMENT, "standard view postprocess scalars must be finite",
                            error_text, error_capacity);
            }
            if (pixels > static_cast<uint64_t>(INT_MAX)) {
                return fail(HS_STATUS_RANGE_ERROR, "postprocess_camera pixel count exceeds cuBLAS int range",
                            error_text, error_capacity);
            }
            if (v->pixel_rays3 == nullptr || v->rgb_map3 == nullptr || v->acc_map == nullptr ||
                v->dpt_map == nullptr || v->norm_map3 == nullptr || v->surf_norm_map3 == nullptr ||
                v->dist_map == nullptr || v->spec_map == nullptr || v->rough_map == nullptr) {
                return fail(HS_STATUS_INVALID_ARGUMENT, "standard view postprocess received a null buffer",
                            error_text, error_capacity);
            }
        }
        // every argument is checked; only now are the handles read
        if (contexts[0]->device != contexts[1]->device) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "standard view handles must be of one device", error_text,
                        error_capacity);
        }
        const int32_t ds = select_device(contexts[0], error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        HsRasterizerContext* first = contexts[0] < contexts[1] ? contexts[0] : contexts[1];
        HsRasterizerContext* second = contexts[0] < contexts[1] ? contexts[1] : contexts[0];
        std::lock_guard<std::mutex> lock_first(first->mutex);
        std::lock_guard<std::mutex> lock_second(second->mutex);
        HsRasterizerContext* base = contexts[0];
        HsRasterizerContext* refl = contexts[1];
        if (post && (base->math_workspace == nullptr || base->math_solver == nullptr ||
                     base->math_tf32_blas == nullptr)) {
            return fail(HS_STATUS_INTERNAL_ERROR, "postprocess_camera math context is not initialized",
                        error_text, error_capacity);
        }
        if (v->trace == 1 && refl->tr_triangles == 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX scene is not built", error_text, error_capacity);
        }
        const cudaStream_t s = static_cast<cudaStream_t>(v->stream);
        const bool traced = v->trace == 1;
        // Queues the whole view on s. captured: inside a stream capture of s,
        // with the raster calls sized for their pair capacities: nothing
        // waits on the host, and a branch after both calls' binning publishes
        // their status for the host (signal_event).
        auto queue_view = [&](const hs::StandardCall* view_calls, bool captured) -> int32_t {
            cudaError_t e = cudaSuccess;
            // postprocess camera terms: only the camera, so beside everything else
            if (post) {
                e = hs::ensure_post_stream(base);
                if (e == cudaSuccess) e = cudaEventRecord(base->post_fork_event, s);
                if (e == cudaSuccess) e = cudaStreamWaitEvent(base->post_stream, base->post_fork_event, 0);
                if (e != cudaSuccess) return cuda_failure(e, "standard view fork", error_text, error_capacity);
                const int32_t ps = camera_terms(base, v->width, v->height, v->fov_x, v->fov_y, v->viewmatrix4x4,
                                                v->camera30, v->pixel_rays3, base->post_stream, error_text,
                                                error_capacity, captured);
                if (ps != HS_STATUS_OK) return ps;
                e = cudaEventRecord(base->post_done_event, base->post_stream);
                if (e != cudaSuccess) return cuda_failure(e, "standard view join", error_text, error_capacity);
            }
            // base colours, and the reflection's prefix, normal column, suffix and
            // (traced) ray split or (untraced) colours, side by side in one grid
            e = hs::precise::view_prologue(
                v->base_sh, v->sh_coefficients, v->sh_degree, v->base.means3d, v->camera_position3, v->base.specular,
                v->base.roughness, nb, v->base.colors5, v->reflection_rotation_raw4, v->reflection.means3d, nr,
                v->reflection_rotation9, v->reflection_normal3, v->reflection_rays36,
                traced ? v->reflection_ray_origins3 : nullptr, traced ? v->reflection_ray_directions3 : nullptr,
                v->reflection_rgb3, v->reflection.specular, v->reflection.roughness,
                traced ? nullptr : v->reflection.colors5, s);
            if (e != cudaSuccess) return cuda_failure(e, "standard view preparation", error_text, error_capacity);
            if (traced && nr != 0) {
                const hs::TraceCall t = view_trace_call(*v, nr, v->reflection.means3d, v->reflection_shs,
                                                        v->reflection_others2, v->reflection.opacities,
                                                        v->reflection.scales2, v->reflection.rotations4,
                                                        v->viewmatrix4x4, v->projmatrix4x4, v->camera_position3, s);
                e = hs::trace_rays(refl, t);
                if (e != cudaSuccess) return cuda_failure(e, "reflection trace", error_text, error_capacity);
                e = hs::view::colors5(v->trace_rgb3, v->reflection.specular, v->reflection.roughness, nr,
                                      v->reflection.colors5, s);
                if (e != cudaSuccess) return cuda_failure(e, "standard view colours", error_text, error_capacity);
            }
            // both raster calls, concurrently
            if (captured) {
                e = hs::standard_forward_many(contexts, view_calls, 2, s, base->graph_fork_event, false);
                const uint64_t counts[2] = {nb, nr};
                if (e == cudaSuccess) e = cudaStreamWaitEvent(base->signal_stream, base->graph_fork_event, 0);
                if (e == cudaSuccess) e = hs::standard_view_status(contexts, counts, 2, base->signal_stream);
                if (e == cudaSuccess)
                    e = cudaEventRecordWithFlags(base->signal_event, base->signal_stream, cudaEventRecordExternal);
                if (e == cudaSuccess) e = cudaEventRecord(base->graph_join_event, base->signal_stream);
                if (e == cudaSuccess) e = cudaStreamWaitEvent(s, base->graph_join_event, 0);
            } else {
                e = hs::standard_forward_many(contexts, view_calls, 2, s,
                                              static_cast<cudaEvent_t>(v->raster_begin_event));
            }
            if (e != cudaSuccess)
                return cuda_failure(e, "concurrent five-channel rasterizer forward", error_text, error_capacity);
            // fusion from the colour planes (renderer.py:326, math.py:301-311) and,
            // with the postprocess, the maps in the same pass
            if (post) {
                e = cudaStreamWaitEvent(s, base->post_done_event, 0);
                if (e != cudaSuccess) return cuda_failure(e, "standard view join", error_text, error_capacity);
                // (1 - ratio) and ratio as float32 scalars of a double ratio (math.py:440-442)
                const float keep = static_cast<float>(1.0 - v->depth_ratio);
                const float ratio = static_cast<float>(v->depth_ratio);
                const hs::post::StandardMaps maps{v->rgb_map3, v->acc_map, v->dpt_map, v->norm_map3,
                                                 v->surf_norm_map3, v->dist_map, v->spec_map, v->rough_map};
                e = hs::post::standard_with_fusion(v->width, v->height, v->base.output_color5, v->base.output_aux7,
                                                   v->pixel_rays3, v->camera30 + 18, v->camera30 + 21, keep, ratio,
                                                   maps, v->reflection.output_color5, v->diffuse_rgb3, v->fused_rgb3,
                                                   v->reflection_rgb_map3, s);
                if (e != cudaSuccess) return cuda_failure(e, "standard view postprocess", error_text, error_capacity);
            } else {
                e = hs::precise::fuse_maps_planar(v->base.output_color5, v->reflection.output_color5,
                                                  v->base.output_color5 + 3 * pixels, v->diffuse_rgb3, v->fused_rgb3,
                                                  v->reflection_rgb_map3, pixels, s);
                if (e != cudaSuccess) return cuda_failure(e, "standard view fusion", error_text, error_capacity);
            }
            const cudaError_t trailing = cudaGetLastError();
            if (trailing != cudaSuccess)
                return cuda_failure(trailing, "standard view execution", error_text, error_capacity);
            return HS_STATUS_OK;
        };
        auto direct = [&]() -> int32_t {
            const int32_t qs = queue_view(calls, false);
            return qs != HS_STATUS_OK ? qs : ok(error_text, error_capacity);
        };
        // Graph replays: a view whose arguments and buffers repeat those of
        // a recent call is captured once and then replayed as one graph
        // launch (no launch of its own per kernel, no host wait before the
        // renderers). Each raster call is captured for a pair capacity an
        // eighth (plus 16384) above the largest of its context's last 16
        // pair counts; a replay whose count exceeds it (or that breaks a
        // limit the direct path checks) is rendered again directly, which
        // grows the buffers and reports what the direct path reports.
        const bool replayable = !traced && v->raster_begin_event == nullptr && nb != 0 && nr != 0 &&
                                view_graphs_enabled() && !base->timer.enabled && !refl->timer.enabled &&
                                base->test_stall_tile == UINT32_MAX && refl->test_stall_tile == UINT32_MAX &&
                                base->std_last_emitted != 0 && refl->std_last_emitted != 0;
        if (!replayable) return direct();
        std::vector<unsigned char> key = view_graph_key(v, sizeof(HsB200StandardViewV2), contexts, 2);
        HsRasterizerContext::ViewGraph* g = find_view_graph(base, key);
        bool captured_now = false;  // the capture itself counted the camera terms' library calls
        if (g == nullptr) {
            // seen once: remember the key (the last few, so that views cycling
            // through a few output buffers replay too) and render directly
            auto& recent = base->view_recent_keys;
            const auto seen = std::find(recent.begin(), recent.end(), key);
            if (seen == recent.end()) {
                if (recent.size() >= 2 * kMaxViewGraphs) recent.erase(recent.begin());
                recent.push_back(std::move(key));
                return direct();
            }
            recent.erase(seen);
            cudaError_t e = hs::ensure_graph_streams(base);
            uint32_t capacity[2];
            for (int i = 0; i < 2; ++i) {
                HsRasterizerContext* c = contexts[i];
                if (e == cudaSuccess) e = hs::ensure_side_stream(c);
                const uint64_t recent = hs::recent_standard_pairs(c);
                capacity[i] = static_cast<uint32_t>(
                    std::min<uint64_t>(recent + recent / 8 + 16384, hs::kMaxStandardPairs));
                if (e == cudaSuccess && hs::standard_pair_capacity(c) < capacity[i])
                    e = hs::standard_reserve_pairs(c, capacity[i]);
            }
            if (e == cudaSuccess && post) e = hs::ensure_post_stream(base);
            if (e != cudaSuccess) return cuda_failure(e, "standard view graph setup", error_text, error_capacity);
            // the grids are sized for the capacity, not for the (larger) buffers
            hs::StandardCall graph_calls[2] = {calls[0], calls[1]};
            for (int i = 0; i < 2; ++i) graph_calls[i].pair_capacity = capacity[i];
            const cudaGraphExec_t exec = capture_view(
                s, [&]() { return queue_view(graph_calls, true) == HS_STATUS_OK; },
                {base->post_stream, base->signal_stream, base->side_stream, refl->side_stream},
                base->graph_join_event);
            ++base->view_graph_captures;
            captured_now = true;
            // the key of the buffers as captured (the reservation may have grown them)
            g = insert_view_graph(base, view_graph_key(v, sizeof(HsB200StandardViewV2), contexts, 2), exec,
                                  capacity);
        }
        if (g->exec == nullptr) return direct();
        g->last_use = ++base->view_graph_clock;
        cudaError_t e = cudaSuccess;
        // the camera terms' workspace: after its previous user, as the direct path orders it
        if (post) e = cudaStreamWaitEvent(s, base->view_camera_event, 0);
        if (e == cudaSuccess) e = cudaGraphLaunch(g->exec, s);
        if (e == cudaSuccess && post) e = cudaEventRecord(base->view_camera_event, s);
        if (e != cudaSuccess) return cuda_failure(e, "standard view graph launch", error_text, error_capacity);
        ++base->view_graph_replays;
        if (post && !captured_now) {
            base->math_matmul_calls += 2;
            base->math_general_inverse_calls += 2;
        }
        // The end of both calls' binning, with the renderers queued (the
        // direct path's finish()).
        e = cudaEventSynchronize(base->signal_event);
        if (e != cudaSuccess) return cuda_failure(e, "standard view graph status", error_text, error_capacity);
        bool gave_up = false, again = false;
        for (int i = 0; i < 2; ++i) {
            const uint32_t* t = contexts[i]->std_total_host;
            gave_up = gave_up || t[3] != 0;
            again = again || t[1] != 0 || t[0] > static_cast<uint32_t>(INT_MAX) || t[2] > g->capacity[i];
            hs::note_standard_pairs(contexts[i], t[2]);
        }
        if (gave_up) {
            return cuda_failure(hs::kWaitGaveUp, "concurrent five-channel rasterizer forward", error_text,
                                error_capacity);
        }
        if (again) {
            ++base->view_graph_reruns;
            return direct();
        }
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_flashgs_view_v2(const HsB200FlashgsViewV2* v, char* error_text,
                                uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (v == nullptr || v->struct_size < sizeof(HsB200FlashgsViewV2)) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS view is null or its struct_size is too small",
                        error_text, error_capacity);
        }
        const bool traced = v->trace == 1;
        // the two raster calls, checked as the concurrent entry checks them;
        // traced, the reflection call takes the trace's colours
        HsB200FlashgsCallV2 refl_args = v->reflection;
        if (traced) refl_args.colors3 = v->trace_rgb3;
        hs::FlashgsCall calls[2];
        int32_t cs = check_flashgs(v->base, &calls[0], error_text, error_capacity);
        if (cs == HS_STATUS_OK) cs = check_flashgs(refl_args, &calls[1], error_text, error_capacity);
        if (cs != HS_STATUS_OK) return cs;
        HsRasterizerContext* contexts[2] = {v->base.handle, v->reflection.handle};
        if (contexts[0] == contexts[1]) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS view needs two distinct handles", error_text,
                        error_capacity);
        }
        if (v->base.use_sh != 1 || v->reflection.use_sh != 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS view takes the base call with SH, the reflection "
                        "call with colours", error_text, error_capacity);
        }
        if (v->base.width != v->reflection.width || v->base.height != v->reflection.height ||
            v->base.tile_row_begin != 0 || v->base.tile_row_end != UINT32_MAX ||
            v->reflection.tile_row_begin != 0 || v->reflection.tile_row_end != UINT32_MAX) {
            return fail(HS_STATUS_RANGE_ERROR, "FlashGS view calls must render the same whole frame", error_text,
                        error_capacity);
        }
        const uint64_t nr = v->reflection.point_count;
        if ((nr != 0 && (v->trace_means3d == nullptr || v->trace_rotation_raw4 == nullptr ||
                         v->reflection_rotation9 == nullptr || v->reflection_normal3 == nullptr ||
                         v->reflection_rays36 == nullptr)) ||
            v->camera_center3 == nullptr || v->fused_rgb3 == nullptr || v->diffuse_rgb3 == nullptr ||
            v->reflection_rgb_map3 == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS view received a null required buffer", error_text,
                        error_capacity);
        }
        const int32_t ts = check_view_trace(*v, nr, v->trace_shs, v->trace_others2, "FlashGS view", error_text,
                                            error_capacity);
        if (ts != HS_STATUS_OK) return ts;
        if (traced && ((nr != 0 && (v->trace_opacities == nullptr || v->trace_scales2 == nullptr ||
                                    v->trace_rotations4 == nullptr)) ||
                       v->world_view4x4 == nullptr || v->full_proj4x4 == nullptr)) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX trace received a null non-empty buffer", error_text,
                        error_capacity);
        }
        if (v->postprocess != 0 && v->postprocess != 1) {
            return fail(HS_STATUS_RANGE_ERROR, "FlashGS view postprocess must be 0 or 1", error_text,
                        error_capacity);
        }
        if (v->postprocess == 1 && (v->world_view4x4 == nullptr || v->rgb_map3 == nullptr ||
                                    v->acc_map == nullptr || v->dpt_map == nullptr || v->norm_map3 == nullptr ||
                                    v->spec_map == nullptr)) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS view postprocess received a null buffer", error_text,
                        error_capacity);
        }
        // every argument is checked; only now are the handles read
        if (contexts[0]->device != contexts[1]->device) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "FlashGS view handles must be of one device", error_text,
                        error_capacity);
        }
        const int32_t ds = select_device(contexts[0], error_text, error_capacity);
        if (ds != HS_STATUS_OK) return ds;
        HsRasterizerContext* first = contexts[0] < contexts[1] ? contexts[0] : contexts[1];
        HsRasterizerContext* second = contexts[0] < contexts[1] ? contexts[1] : contexts[0];
        std::lock_guard<std::mutex> lock_first(first->mutex);
        std::lock_guard<std::mutex> lock_second(second->mutex);
        HsRasterizerContext* refl = contexts[1];
        if (traced && refl->tr_triangles == 0) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "OptiX scene is not built", error_text, error_capacity);
        }
        const cudaStream_t s = static_cast<cudaStream_t>(v->stream);
        // prefix, normal column, suffix and (traced) the ray split, in one pass
        cudaError_t e = hs::precise::reflection_view(
            v->trace_rotation_raw4, v->trace_means3d, v->camera_center3, nr, v->reflection_rotation9,
            v->reflection_normal3, v->reflection_rays36, traced ? v->reflection_ray_origins3 : nullptr,
            traced ? v->reflection_ray_directions3 : nullptr, nullptr, nullptr, nullptr, nullptr, s);
        if (e != cudaSuccess) return cuda_failure(e, "FlashGS view preparation", error_text, error_capacity);
        if (traced && nr != 0) {
            const hs::TraceCall t = view_trace_call(*v, nr, v->trace_means3d, v->trace_shs, v->trace_others2,
                                                    v->trace_opacities, v->trace_scales2, v->trace_rotations4,
                                                    v->world_view4x4, v->full_proj4x4, v->camera_center3, s);
            e = hs::trace_rays(refl, t);
            if (e != cudaSuccess) return cuda_failure(e, "reflection trace", error_text, error_capacity);
        }
        // both raster calls, concurrently
        e = hs::flashgs_forward_many(contexts, calls, 2, s, static_cast<cudaEvent_t>(v->raster_begin_event));
        if (e != cudaSuccess) return cuda_failure(e, "concurrent FlashGS forward", error_text, error_capacity);
        // fusion from the colour planes; specular is the base call's other[0]
        // (renderer.py:420-427); with the postprocess, in the maps pass
        const uint64_t pixels = static_cast<uint64_t>(v->base.width) * static_cast<uint64_t>(v->base.height);
        if (v->postprocess == 1) {
            const hs::post::FlashgsMaps maps{v->rgb_map3, v->acc_map, v->dpt_map, v->norm_map3,
                                             v->surf_norm_map3, v->dist_map, v->spec_map};
            e = hs::post::flashgs_from_view(v->base.width, v->base.height, v->base.output_color3,
                                            v->base.output_other2, v->base.output_depth1, v->base.output_alpha1,
                                            v->base.output_normal3, v->world_view4x4, maps,
                                            v->reflection.output_color3, v->diffuse_rgb3, v->fused_rgb3,
                                            v->reflection_rgb_map3, s);
            if (e != cudaSuccess) return cuda_failure(e, "FlashGS view postprocess", error_text, error_capacity);
        } else {
            e = hs::precise::fuse_maps_planar(v->base.output_color3, v->reflection.output_color3,
                                              v->base.output_other2, v->diffuse_rgb3, v->fused_rgb3,
                                              v->reflection_rgb_map3, pixels, s);
            if (e != cudaSuccess) return cuda_failure(e, "FlashGS view fusion", error_text, error_capacity);
        }
        const cudaError_t trailing = cudaGetLastError();
        if (trailing != cudaSuccess)
            return cuda_failure(trailing, "FlashGS view execution", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_view_graph_stats_v1(HsRasterizerHandle base_handle, uint64_t* captures, uint64_t* replays,
                                    uint64_t* reruns, char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (base_handle == nullptr || captures == nullptr || replays == nullptr || reruns == nullptr) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "view graph stats received a null pointer", error_text,
                        error_capacity);
        }
        std::lock_guard<std::mutex> lock(base_handle->mutex);
        *captures = base_handle->view_graph_captures;
        *replays = base_handle->view_graph_replays;
        *reruns = base_handle->view_graph_reruns;
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_test_pair_ops_v1(const float* a, const float* b, const float* c, const float* d, uint64_t count,
                                 uint32_t* mismatches16, char* error_text, uint64_t error_capacity) noexcept {
    return guard(error_text, error_capacity, [&]() -> int32_t {
        if (mismatches16 == nullptr || (count >= 2 && (a == nullptr || b == nullptr || c == nullptr || d == nullptr))) {
            return fail(HS_STATUS_INVALID_ARGUMENT, "pair check received a null buffer", error_text, error_capacity);
        }
        const cudaError_t e = hs::pair_check(a, b, c, d, count, mismatches16, nullptr);
        if (e != cudaSuccess) return cuda_failure(e, "pair check", error_text, error_capacity);
        return ok(error_text, error_capacity);
    });
}

int32_t hs_b200_flashgs_forward_many_v2(const HsB200FlashgsCallV2* calls, uint32_t call_count,
                                        void* stream, char* error_text,
                                        uint64_t error_capacity) noexcept {
    return many_entry<HsB200FlashgsCallV2, hs::FlashgsCall>(
        calls, call_count, stream, "concurrent FlashGS forward", check_flashgs,
        [](HsRasterizerContext* const* c, const hs::FlashgsCall* k, uint32_t n, cudaStream_t st) {
            return hs::flashgs_forward_many(c, k, n, st);
        },
        error_text, error_capacity);
}

int32_t hs_b200_rasterizer_forward_many_v2(const HsB200RasterizerCallV2* calls,
                                           uint32_t call_count, void* stream, char* error_text,
                                           uint64_t error_capacity) noexcept {
    return many_entry<HsB200RasterizerCallV2, hs::StandardCall>(
        calls, call_count, stream, "concurrent five-channel rasterizer forward", check_rasterizer,
        [](HsRasterizerContext* const* c, const hs::StandardCall* k, uint32_t n, cudaStream_t st) {
            return hs::standard_forward_many(c, k, n, st);
        },
        error_text, error_capacity);
}

}  // extern "C"
