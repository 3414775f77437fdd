/*
 * msplat_c_api.h — trainer-level C API of the B200 build.
 *
 * Same types and functions as the reference's public C ABI
 * (core/include/msplat_c_api.h:1-133, implemented at
 * core/src/msplat_api.mm:282-407), so callers written against it (the Swift
 * package, demos) keep working. Differences:
 *   - dataset loaders (COLMAP / Nerfstudio / Polycam) are not part of this
 *     build: msplat_dataset_create returns NULL with msplat_last_error() set;
 *     build datasets with msplat_dataset_create_from_memory instead;
 *   - densification runs inside msplat_trainer_step as in Model::afterTrain
 *     (with the scale compaction fixed to 2 floats per row, see
 *     msplat_densify_plan); PLY/.splat export and "MSPL" v1 checkpoints are
 *     byte-compatible with the reference's; a checkpoint whose SH degree
 *     differs from the trainer's is rejected (the reference reads it anyway);
 *   - mesh extraction (TSDF + marching cubes) is not part of this build: the
 *     call records an error and returns -1;
 *   - errors never escape as C++ exceptions: failed calls return NULL / zero
 *     structures and set msplat_last_error() (declared in msplat_backend.h);
 *   - msplat_set_metallib_path is accepted and ignored.
 */
#ifndef MSPLAT_C_API_H
#define MSPLAT_C_API_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── Config (msplat_c_api.h:16-53) ─────────────────────────────────────────── */

typedef struct {
    int iterations;
    int shDegree;
    int shDegreeInterval;
    float ssimWeight;
    int numDownscales;
    int resolutionSchedule;
    int refineEvery;
    int warmupLength;
    int resetAlphaEvery;
    float densifyGradThresh;
    float densifySizeThresh;
    int stopScreenSizeAt;
    float splitScreenSize;
    bool keepCrs;
    float downscaleFactor;
    float bgColor[3];
} MsplatConfig;

static inline MsplatConfig msplat_default_config(void) {
    MsplatConfig c;
    c.iterations = 30000;
    c.shDegree = 3;
    c.shDegreeInterval = 1000;
    c.ssimWeight = 0.2f;
    c.numDownscales = 2;
    c.resolutionSchedule = 3000;
    c.refineEvery = 100;
    c.warmupLength = 500;
    c.resetAlphaEvery = 30;
    c.densifyGradThresh = 0.0002f;
    c.densifySizeThresh = 0.01f;
    c.stopScreenSizeAt = 4000;
    c.splitScreenSize = 0.05f;
    c.keepCrs = false;
    c.downscaleFactor = 1.0f;
    c.bgColor[0] = 0.6130f; c.bgColor[1] = 0.0101f; c.bgColor[2] = 0.3984f;
    return c;
}

/* ── Stats / metrics / pixel buffer (msplat_c_api.h:57-81) ─────────────────── */

typedef struct {
    int iteration;
    int splatCount;
    float msPerStep;
    float loss;
} MsplatStats;

typedef struct {
    float psnr;
    float ssim;
    float l1;
    int numTest;
    int numGaussians;
} MsplatEvalMetrics;

typedef struct {
    float* data;   /* RGB float32, HWC layout. Caller must free() this. */
    int width;
    int height;
} MsplatPixelBuffer;

/* ── Dataset (msplat_c_api.h:85-92) ──────────────────────────────────────── */

typedef void* MsplatDataset;

/* Replaces msplat_dataset_create (msplat_c_api.h:87): file loaders are not
 * part of this build; returns NULL and sets msplat_last_error(). */
MsplatDataset msplat_dataset_create(const char* path, float downscaleFactor, bool evalMode, int testEvery);
void msplat_dataset_destroy(MsplatDataset ds);
int msplat_dataset_num_train(MsplatDataset ds);
int msplat_dataset_num_test(MsplatDataset ds);
void msplat_dataset_camera_pose(MsplatDataset ds, int cameraIndex, float camToWorld[16]);

/* Additive: a dataset from host memory. numCameras OpenGL camToWorld matrices
 * (row-major 4x4 each), intrinsics (fx, fy, cx, cy) per camera, one image
 * size for all cameras, images [numCameras][height][width][3] float32 in
 * [0, 1] (copied into pinned host memory; may be NULL for a render-only
 * dataset), and an initial point cloud (xyz float32, rgb uint8; may be empty).
 * evalMode splits every testEvery-th camera into the test set, as
 * InputData::splitTrainTest does. */
MsplatDataset msplat_dataset_create_from_memory(int numCameras, const float* camToWorld, const float* intrinsics,
                                                int width, int height, const float* images, int numPoints,
                                                const float* xyz, const uint8_t* rgb, bool evalMode,
                                                int testEvery);

/* ── Trainer (msplat_c_api.h:96-124) ─────────────────────────────────────── */

typedef void* MsplatTrainer;

/* Model::Model initialisation from the dataset's point cloud (model.cpp:43-121):
 * log of the mean distance to the 3 nearest neighbours for both scales,
 * random unit quaternions from mt19937(42), DC colour from RGB, zero higher
 * bands, opacity logit(0.1). */
MsplatTrainer msplat_trainer_create(MsplatDataset ds, MsplatConfig config);
/* Additive: start from given parameters (host float32, reference layout:
 * means [N,3], scales [N,2] log, quats [N,4], opacities [N] logit,
 * featuresDc [N,3], featuresRest [N,K,3] with K = (shDegree+1)^2 - 1; may be
 * NULL when K == 0). */
MsplatTrainer msplat_trainer_create_from_params(MsplatDataset ds, MsplatConfig config, int numPoints,
                                                const float* means, const float* scales, const float* quats,
                                                const float* opacities, const float* featuresDc,
                                                const float* featuresRest);
void msplat_trainer_destroy(MsplatTrainer t);

/* Trainer::step (msplat_api.mm:106-128): next shuffled camera (mt19937(42)),
 * its target image copied host->device, one fused training step, means
 * learning-rate schedule, loss read back. */
MsplatStats msplat_trainer_step(MsplatTrainer t);
void msplat_trainer_train(MsplatTrainer t);
MsplatEvalMetrics msplat_trainer_evaluate(MsplatTrainer t);
MsplatPixelBuffer msplat_trainer_render(MsplatTrainer t, int cameraIndex, bool useTest);
MsplatPixelBuffer msplat_trainer_render_pose(MsplatTrainer t, const float camToWorld[16], int refCameraIndex);
void msplat_trainer_render_pose_to_buffer(MsplatTrainer t, const float camToWorld[16], int refCameraIndex,
                                          uint8_t* outRGBA, int* outWidth, int* outHeight);
void msplat_trainer_export_ply(MsplatTrainer t, const char* path);
void msplat_trainer_export_splat(MsplatTrainer t, const char* path);
int64_t msplat_trainer_extract_mesh(MsplatTrainer t, const char* path, float voxelSize, float boundRadius,
                                    float alphaThresh, float truncMultiplier);
void msplat_trainer_save_checkpoint(MsplatTrainer t, const char* path);
int msplat_trainer_load_checkpoint(MsplatTrainer t, const char* path);
int msplat_trainer_splat_count(MsplatTrainer t);
int msplat_trainer_iteration(MsplatTrainer t);

/* Additive: copies the current parameters to host arrays (reference layout;
 * any pointer may be NULL). Returns 0 on success. */
int msplat_trainer_get_params(MsplatTrainer t, float* means, float* scales, float* quats, float* opacities,
                              float* featuresDc, float* featuresRest);

/* Additive: when enable != 0, every later msplat_trainer_step also writes the
 * per-group gradients it hands to Adam (the tensors Model::fullIteration
 * passes to its six msplat_fused_adam calls, core/src/model.cpp:800-826) to
 * the backend workspace, readable with msplat_last_tensor (dL_dmean3D,
 * dL_dscale, dL_dquat, dL_dfeatures_dc, dL_dfeatures_rest, dL_dopacity)
 * until the next backend call on the device. Costs one extra write of every
 * gradient per step. Returns 0 on success. */
int msplat_trainer_set_write_gradients(MsplatTrainer t, int enable);

/* ── Lifecycle (msplat_c_api.h:126-130) ──────────────────────────────────── */

void msplat_set_metallib_path(const char* path);
void msplat_sync(void);
void msplat_cleanup(void);

#ifdef __cplusplus
}
#endif

#endif /* MSPLAT_C_API_H */
