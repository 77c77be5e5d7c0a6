/*
 * gofish_b200: C ABI of the B200 (sm_100a) fisheye Gaussian tracer.
 *
 * Plain pointers and sizes only.  Every device pointer is CUDA global memory
 * on the device that is current when the call is made; `stream` is a
 * cudaStream_t passed as void*.  All work is enqueued on that stream.  Calls
 * return 0 on success and a negative GF_ERR_* code on failure, in which case
 * gf_last_error() describes the failure (thread-local string).
 *
 * Each entry point replaces one method of the reference's pybind module
 * (tuallen/GOFish, threedgut_tracer/bindings.cpp:106-165 and
 * src/splatRaster.cpp).
 */
#ifndef GOFISH_B200_H
#define GOFISH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GF_ABI_VERSION 7

#define GF_OK 0
#define GF_ERR_BAD_INPUT (-1)
#define GF_ERR_CUDA (-2)
#define GF_ERR_NOT_REGISTERED (-3)
#define GF_ERR_STATE (-4)
#define GF_ERR_CAPACITY (-5)

/* Camera model types (cameraModels.h ModelType) and shutter types
 * (cameraModels.h:51-57 ShutterType; only GLOBAL is rendered, as in the
 * reference, gutRenderer.cu:704-706). */
#define GF_CAMERA_OPENCV_PINHOLE 0
#define GF_CAMERA_OPENCV_FISHEYE 1
#define GF_SHUTTER_ROLLING_TOP_TO_BOTTOM 0
#define GF_SHUTTER_ROLLING_LEFT_TO_RIGHT 1
#define GF_SHUTTER_ROLLING_BOTTOM_TO_TOP 2
#define GF_SHUTTER_ROLLING_RIGHT_TO_LEFT 3
#define GF_SHUTTER_GLOBAL 4

/* Camera model parameters.  Replaces the TSensorModel built by
 * fromOpenCVFisheyeCameraModelParameters / fromOpenCVPinholeCameraModelParameters
 * (threedgut_tracer/bindings.cpp:36-79).  Fisheye uses radial[0..3] = k1..k4
 * and max_angle; pinhole uses radial[0..5], tangential and thin_prism. */
typedef struct gf_camera {
    int32_t model;
    int32_t width;
    int32_t height;
    int32_t shutter;
    float principal_point[2];
    float focal_length[2];
    float radial[6];
    float tangential[2];
    float thin_prism[4];
    float max_angle;
    float reserved;
} gf_camera;

/* Sort key of the (tile | depth) radix sort. */
#define GF_KEY_PER_TILE_DEPTH 0  /* per-tile maximum-response depth (gutProjector.cuh:364-417) */
#define GF_KEY_GLOBAL_DEPTH 1    /* camera radial distance (gutProjector.cuh:426-427)           */

/* Renderer configuration.  Replaces SplatRaster(json conf) (bindings.cpp:109)
 * for the settings that change this path: render.splat.k_buffer_size,
 * render.gofish.fast_global_depth_key and render.enable_hitcounts. */
typedef struct gf_tracer_config {
    int32_t k_buffer_size;     /* 0, 4, 8, 12, 16, 24 or 32 */
    int32_t sort_key;          /* GF_KEY_* */
    int32_t enable_hit_counts; /* 1: write the per-pixel hit count */
    int32_t admission_fallback; /* GF_FALLBACK_*: admission of particles without a valid projection */
    int32_t composite_log_capacity; /* entries per pixel of the training forward's composite log, read by the
                                       backward: 0 = default (256), < 0 = no log (the backward replays every
                                       tile through the k-buffer) */
    int32_t enable_normals;         /* render.enable_normals: 1 computes the geometric training channels
                                       (gf_trace_outputs.normal ... inv_depth2) and their gradients */
    int32_t intersection_capacity;  /* GF_CAPACITY_*: how the tile-intersection keys are sized */
    int32_t compositor;             /* GF_COMPOSITOR_*: render.splat.hierarchical_sort */
    int32_t complete_admission;     /* render.gofish.complete_admission: 1 admits every particle (density >= 1/255)
                                       by the conservative cone test of its support sphere, whose tiles hold every
                                       pixel its hit test can pass on; 0 admits particles with a valid unscented
                                       projection by their footprint (admission_fallback for the others) */
    float fallback_min_angle;       /* GF_FALLBACK_CONE_BIG: half-angle window [min, max] (radians, 0 <= min <= max)
                                       of the caps the fallback admits (render.gofish.fast_admission_fallback_
                                       {min,max}_angle_deg, setup_3dgut.py:235-239) */
    float fallback_max_angle;
    float partial_ut_scale;         /* render.gofish.fast_partial_ut_scale (gutProjector.cuh:53-62, :470-499): > 0
                                       repairs a projection whose mean is valid and whose every axis keeps one
                                       valid sigma point (each invalid point replaced by the reflection of its
                                       mirror about the projected mean, the covariance scaled by its square);
                                       0 = off (every sigma point must project) */
} gf_tracer_config;

/* Compositing order of a pixel's hits.  KBUFFER: the tile's depth-sorted
 * candidates through a per-pixel k-buffer of k_buffer_size
 * (gutKBufferRenderer.cuh:614-700).  SOF: SOF's hierarchy, a per-pixel HEAD
 * of 4 fed by per-2x2 MID8 and per-4x4 TAIL64 windows ordered by
 * representative depth (sofMid8Hierarchy.inl:161-598); k_buffer_size is not
 * used. */
#define GF_COMPOSITOR_KBUFFER 0
#define GF_COMPOSITOR_SOF 1

/* Sizing of the tile-intersection keys of a forward.  SPECULATIVE: 1.5x the
 * largest count of the earlier forwards, with no host synchronization (the
 * first forward and any forward whose particle count or raster changed read
 * the exact count); a forward whose count exceeds it renders nothing and the
 * next call on the tracer returns GF_ERR_CAPACITY, with the capacity grown.
 * EXACT: every forward reads its count with one synchronization. */
#define GF_CAPACITY_SPECULATIVE 0
#define GF_CAPACITY_EXACT 1

/* render.gofish.fast_admission_fallback (setup_3dgut.py:232-239): "none"
 * drops particles whose unscented projection is invalid; "cone" admits them
 * by their bounding sphere against the tile ray cones; "cone_big" does so
 * only for spheres that leave the camera centre outside and whose cap
 * half-angle lies in [fallback_min_angle, fallback_max_angle]
 * (gutProjector.cuh:44-50, :145-154): large UT-invalid particles near the
 * camera, not the many small ones beyond a wide-angle rim. */
#define GF_FALLBACK_NONE 0
#define GF_FALLBACK_CONE 1
#define GF_FALLBACK_CONE_BIG 5

/* Per-call inputs of trace / trace_bwd / trace_inference
 * (splatRaster.cpp:259-273, :383-393, :469-500). */
typedef struct gf_trace_inputs {
    uint32_t frame;
    int32_t sh_degree;          /* active SH degree, 0..3 (n_active_features) */
    uint32_t num_particles;     /* N */
    uint32_t sh_coeffs;         /* coefficients per colour channel in `features`: 1, 4, 9 or 16 */
    const float* particles;     /* device [N,32] packed particle rows (tracer.py:171-179) */
    const float* features;      /* device [N, 3*sh_coeffs] SH coefficients */
    const float* ray_origin;    /* device [H,W,3] sensor-frame ray origins */
    const float* ray_direction; /* device [H,W,3] sensor-frame unit ray directions */
    gf_camera camera;           /* width/height must match the ray grid */
    float pose_start[7];        /* world->sensor [tx,ty,tz,qx,qy,qz,qw] at t0 */
    float pose_end[7];          /* world->sensor pose at t1 (must equal pose_start) */
    int64_t timestamp_start;
    int64_t timestamp_end;
    const char* tile_token;     /* token of a registered physical tile mask */
    int32_t sof_opacity_active; /* sof_exact_opacity_active: trace writes the SOF opacity field (needs
                                   enable_normals, for the exact 0.5-crossing depth) */
} gf_trace_inputs;

/* Forward outputs (caller-allocated device buffers, initialized by the call
 * exactly as splatRaster.cpp:293-313 initializes its tensors). */
typedef struct gf_trace_outputs {
    float* rgba;          /* [H,W,4] radiance + opacity                       */
    float* hit_distance;  /* [H,W,1]                                           */
    float* hit_count;     /* [H,W,1] or NULL                                   */
    float* visibility;    /* [N,1]: int bit pattern 1 where the particle is admitted to a tile, else 0; or NULL */
    /* Geometric training channels (rayPayload.cuh:242-322), written when the
     * tracer was created with enable_normals; each may be NULL. */
    float* normal;        /* [H,W,3] sum_i w_i n_i, n_i = -normalize(B^-T normalize(B^-1 d)) */
    float* depth_var;     /* [H,W,1] sum_i w_i t_i^2 */
    float* quant;         /* [H,W,10] depths where the accumulated opacity first reaches 0.05, 0.10, 0.15,
                             0.20, 0.30, 0.40, 0.50; the largest-weight hit's depth; the exact 0.5-crossing
                             depth and its opacity rate */
    float* extent;        /* [H,W,1] sum_i w_i sigma_i, sigma_i = |s_i * (R_i^T d)| of the intrinsic shape */
    float* inv_depth;     /* [H,W,1] sum_i w_i / max(d_i, 0.2) */
    float* inv_depth2;    /* [H,W,1] sum_i w_i / max(d_i, 0.2)^2 */
    float* opacity_field; /* [H,W,1] SOF opacity field (gutRenderer.cuh:297-346): 1 - prod(1 - alpha_i) over the
                             tile's candidates, alpha_i of the intrinsic Gaussian (rotation, scale and density of
                             slots 4-11) on the ray up to the exact 0.5 crossing (the whole ray without one);
                             written when sof_opacity_active */
} gf_trace_outputs;

/* Backward inputs/outputs (splatRaster.cpp:469-640). */
typedef struct gf_trace_grads {
    const float* rgba;              /* forward [H,W,4] */
    const float* hit_distance;      /* forward [H,W,1] */
    const float* grad_rgba;         /* dL/d rgba [H,W,4] */
    const float* grad_hit_distance; /* dL/d hit distance [H,W,1] */
    float* grad_particles;          /* out [N,32] (overwritten) */
    float* grad_features;           /* out [N, 3*sh_coeffs] (overwritten) */
    /* Geometric channels (enable_normals): forward values and their
     * gradients, NULL pairs for channels without a gradient.  The extent's
     * gradient reaches the rotation and scale slots (4-10) of grad_particles. */
    const float* normal;
    const float* grad_normal;
    const float* depth_var;
    const float* grad_depth_var;
    const float* extent;
    const float* grad_extent;
    const float* inv_depth;
    const float* grad_inv_depth;
    const float* inv_depth2;
    const float* grad_inv_depth2;
    /* SOF opacity field and its gradient (gutRenderer.cuh:351-430), with the
     * forward's quantile channel (its exact crossing depth); the gradient
     * reaches the position, rotation, scale and intrinsic density slots. */
    const float* quant;
    const float* opacity_field;
    const float* grad_opacity_field;
    /* dL/d quant [H,W,10] (with quant): the exact 0.5-crossing depth's channel
     * (8) back-propagates by the implicit function theorem through the hits
     * before the crossing and the crossing Gaussian evaluated at that depth
     * (gaussianParticles.cuh:934-986, rayPayloadBackward.cuh:122-128); the other
     * channels carry no gradient.  NULL: no crossing gradient. */
    const float* grad_quant;
    /* Densification statistic (splatRaster.cpp:515-531,628-649 with
     * gutKBufferRenderer.cuh:283-296; read by threedgrut/strategy/gs.py:88-96,
     * 306-313): for every composited hit, the absolute value of that hit's
     * position gradient, summed per particle.  NULL: not accumulated.
     * GF_ABS_GRAD_SCREEN: [N,8] floats, slots 0-5 the caller's map M (2x3
     * row-major) of the particle, slots 6 and 7 += |M[0,:] g| and |M[1,:] g|.
     * GF_ABS_GRAD_WORLD: [N,3] floats += |g_x|, |g_y|, |g_z|. */
    float* position_abs_grad;
    int32_t position_abs_grad_mode;
} gf_trace_grads;

#define GF_ABS_GRAD_SCREEN 1
#define GF_ABS_GRAD_WORLD 2

/* Counters of the last forward pass. */
typedef struct gf_trace_stats {
    uint64_t num_intersections; /* emitted (tile, particle) pairs */
    uint32_t num_tiles;
    uint32_t num_particles;
    uint32_t kernel_launches;   /* kernels launched by the last trace/trace_bwd call */
    uint32_t fallback_particles; /* particles without a UT footprint handed to the cone admission */
    uint64_t total_kernel_launches; /* kernels launched by this tracer since its creation */
    uint64_t total_forwards;        /* forwards since the tracer's creation */
    uint64_t total_intersections;   /* their tile intersections, summed */
    uint64_t total_fallback_particles; /* their cone-fallback particles, summed */
    uint64_t total_host_wait_us;    /* microseconds the calling threads spent waiting for the device */
} gf_trace_stats;

typedef struct gf_tracer gf_tracer;

/* Library ABI version (GF_ABI_VERSION). */
int gf_abi_version(void);

/* Thread-local description of the last error. */
const char* gf_last_error(void);

/* SplatRaster::SplatRaster(json) -- bindings.cpp:109, splatRaster.cpp:106-153. */
gf_tracer* gf_tracer_create(const gf_tracer_config* config);

/* ~SplatRaster. Frees every device buffer the tracer owns. */
void gf_tracer_destroy(gf_tracer* tracer);

/* SplatRaster::registerPhysicalTileMask -- bindings.cpp:123, splatRaster.cpp:229-248.
 * `mask` is a device uint8 [tiles_y, tiles_x] array; it is copied. */
int gf_tracer_register_tile_mask(gf_tracer* tracer, const uint8_t* mask, uint32_t tiles_y, uint32_t tiles_x,
                                 const char* token, void* stream);

/* SplatRaster::trace -- bindings.cpp:110, splatRaster.cpp:259-380 (colour,
 * opacity, hit distance, hit count and visibility channels). */
int gf_tracer_trace(gf_tracer* tracer, const gf_trace_inputs* inputs, const gf_trace_outputs* outputs,
                    void* stream);

/* SplatRaster::traceBwd -- bindings.cpp:111, splatRaster.cpp:469-640.  Must
 * follow a gf_tracer_trace with the same inputs on the same stream. */
int gf_tracer_trace_bwd(gf_tracer* tracer, const gf_trace_inputs* inputs, const gf_trace_grads* grads,
                        void* stream);

/* SplatRaster::traceInference -- bindings.cpp:113, splatRaster.cpp:383-466. */
int gf_tracer_trace_inference(gf_tracer* tracer, const gf_trace_inputs* inputs, float* rgba, float* hit_distance,
                              void* stream);

/* Stages timed by gf_tracer_collect_times. */
#define GF_STAGE_TILE_RAYS 0
#define GF_STAGE_PROJECT 1
#define GF_STAGE_SCAN 2
#define GF_STAGE_EMIT 3
#define GF_STAGE_SORT 4
#define GF_STAGE_RANGES 5
#define GF_STAGE_RENDER_FWD 6
#define GF_STAGE_RENDER_BWD 7
#define GF_STAGE_PROJECT_BWD 8
#define GF_NUM_STAGES 9

/* Turns per-stage CUDA-event timing on or off (render.enable_kernel_timings,
 * splatRaster.cpp:155-198).  Events are recorded on the call's stream. */
int gf_tracer_enable_timing(gf_tracer* tracer, int enable);

/* SplatRaster::collectTimes (splatRaster.cpp:702-732): writes the summed
 * milliseconds and the launch count of every stage timed since the last
 * collection into ms[GF_NUM_STAGES] and launches[GF_NUM_STAGES] (either may
 * be NULL), then clears them.  Waits for the recorded events. */
int gf_tracer_collect_times(gf_tracer* tracer, float* ms, uint32_t* launches);

/* Counters of the last forward pass (SplatRaster::collectTimes, splatRaster.cpp:702-732, reports timings;
 * this reports the sizes the timings depend on). */
int gf_tracer_stats(const gf_tracer* tracer, gf_trace_stats* stats);

/* Tiles of the last training forward holding a pixel that composited more
 * hits than the composite log holds (0 without a log); trace_bwd replays
 * them through the k-buffer (renderBackward, gutRenderer.cuh:555-712).
 * Waits for that forward's render to finish. */
int gf_tracer_log_overflow_tiles(const gf_tracer* tracer, uint32_t* tiles);

/* Copies the last forward pass's intermediate state into caller device
 * buffers (any pointer may be NULL): projected particle state [N,8]
 * (center.xy, conic.xyz, opacity, extent.xy), precomputed radiance [N,3],
 * per-particle tile counts [N], sorted (tile|depth) keys and particle ids
 * [capacity], and per-tile [begin,end) ranges [T,2].  No reference
 * counterpart: it exposes GutRenderForwardContext (gutRenderer.cu:229-671)
 * for parity tests. */
int gf_tracer_copy_intermediates(const gf_tracer* tracer, float* projected, float* radiance, uint32_t* counts,
                                 uint64_t* sorted_keys, uint32_t* sorted_ids, uint64_t capacity, uint32_t* ranges,
                                 void* stream);

/* Largest number of (key, id) pairs gf_sort_tile_keys_static accepts. */
#define GF_STATIC_SORT_MAX_PAIRS 262144u

/* Stable sort of (tile << 32 | depth bits) keys and their particle ids by the
 * key bits [0, end_bit), the same order as the sort inside gf_tracer_trace.
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory while they render -- hosts that give the library a fixed
 * device budget and forbid allocation on the frame path, real-time loops in
 * which a cudaMalloc (which can synchronize the device) would stall a frame,
 * tools that only pass preallocated buffers.  It allocates nothing: its scratch is a fixed
 * file-scope device array sized for GF_STATIC_SORT_MAX_PAIRS pairs (about
 * 3.1 MiB, held by every GPU that loads the library until exit).  Larger
 * inputs are rejected with GF_ERR_CAPACITY.  The first call on a device
 * resolves the array's device address and must come before any stream
 * capture; the address is kept for the life of the process, so
 * cudaDeviceReset is not supported while the library is loaded.  A CUDA error
 * left by earlier work is returned as GF_ERR_CUDA before anything is launched.
 * All calls on a device share the array: calls whose GPU work
 * overlaps race and must be serialized by the caller.  Inputs are read only
 * and must not alias the outputs. */
int gf_sort_tile_keys_static(const uint64_t* keys_in, const uint32_t* ids_in, uint64_t* keys_out, uint32_t* ids_out,
                             uint32_t n, int end_bit, void* stream);

/* ------------------------------------------------------------------------
 * Mesh opacity field.  Replaces the reference's mesh SplatRaster methods
 * (gofish/mesh/native/bindings.cpp:84-114, implemented in
 * gofish/mesh/native/include/3dgut/kernels/cuda/common/opacityFieldBinding.inl).
 *
 * O_v(x) = 1 - prod(1 - alpha_i) over every Gaussian i whose hit test passes
 * on the segment from camera v's centre to x, in ascending Gaussian id; the
 * field is the minimum of O_v over the cameras that observe x (x projects
 * into the raster, onto an unmasked pixel, at a positive range).
 * ------------------------------------------------------------------------ */

/* One camera: the arguments of integrate_opacity_field_camera and
 * stage_bisection_camera (bindings.cpp:87-105).  Global shutter only, with
 * identical finite start and end poses (opacityFieldBinding.inl:170-196).
 * Every pixel's ray origin must be the same point (one camera centre per
 * view); a point that lands on a pixel with another origin makes
 * gf_field_finish / gf_field_evaluate_round fail. */
typedef struct gf_field_camera {
    uint32_t frame_number;
    uint32_t reserved0;
    gf_camera camera;            /* width x height is the ray raster */
    const float* ray_origin;     /* device [H,W,3], sensor frame */
    const uint8_t* pixel_mask;   /* device [H,W] physical-domain mask, or NULL */
    int64_t timestamp_start;
    int64_t timestamp_end;
    float pose_start[7];         /* world -> sensor [t, q(x,y,z,w)] */
    float pose_end[7];
} gf_field_camera;

typedef struct gf_field gf_field;

typedef struct gf_field_stats {
    uint64_t evaluations;      /* (point, camera) evaluations integrated so far */
    uint64_t pairs;            /* (cell, Gaussian) candidate pairs so far */
    uint64_t cameras;          /* camera passes so far */
    uint64_t kernel_launches;  /* kernels launched so far */
    uint64_t candidate_loads;  /* candidates staged by the integration blocks so far */
    uint64_t hit_tests;        /* exact per-point hit tests so far */
    uint64_t hits;             /* accepted hits so far */
    uint64_t warp_iterations;  /* (warp, candidate) steps of the integration so far */
} gf_field_stats;

/* Stages of a camera pass, for gf_field_collect_times. */
#define GF_FIELD_STAGE_POINTS 0     /* project, key, counting sort of the points */
#define GF_FIELD_STAGE_CONES 1      /* cell cones, quadtree, block counts */
#define GF_FIELD_STAGE_CANDIDATES 2 /* per-Gaussian caps and cell counts, scan */
#define GF_FIELD_STAGE_SORT 3       /* emit, cell-key sort, cell ranges */
#define GF_FIELD_STAGE_INTEGRATE 4  /* ordered integration */
#define GF_FIELD_STAGE_FINISH 5     /* finish / round decision vectors */
#define GF_FIELD_STAGES 6

gf_field* gf_field_create(void);
void gf_field_destroy(gf_field* field);

/* begin_opacity_field (opacityFieldBinding.inl:203-268): copies the packed
 * Gaussians [N,32] (positions 0-2, density 3, B^-1 row-major 21-29) and the
 * query points [Q,3]; sigma_max [N] is validated but the support bound is
 * derived from B^-1 itself.  N > 0, Q > 0.  One context at a time. */
int gf_field_begin(gf_field* field, const float* particles, const float* sigma_max, uint32_t num_particles,
                   const float* points, uint32_t num_points, int64_t* token, void* stream);
/* integrate_opacity_field_camera (opacityFieldBinding.inl:270-316). */
int gf_field_integrate_camera(gf_field* field, int64_t token, const gf_field_camera* camera, void* stream);
/* finish_opacity_field (opacityFieldBinding.inl:318-338): opacity [Q] (0 where
 * unobserved), observed [Q], above [Q] = observed and opacity >= 1/2. */
int gf_field_finish(gf_field* field, int64_t token, float* opacity, uint8_t* observed, uint8_t* above,
                    void* stream);
/* release_opacity_field (opacityFieldBinding.inl:340-347). */
int gf_field_release(gf_field* field, int64_t token, void* stream);

/* begin_bisection_table (opacityFieldBinding.inl:349-368): as gf_field_begin;
 * the probe points fix the round capacity Q. */
int gf_field_begin_table(gf_field* field, const float* particles, const float* sigma_max, uint32_t num_particles,
                         const float* probe_points, uint32_t num_points, int64_t* token, void* stream);
/* stage_bisection_camera (opacityFieldBinding.inl:370-431): copies the
 * camera's ray origins and mask. */
int gf_field_stage_camera(gf_field* field, int64_t token, const gf_field_camera* camera, void* stream);
/* seal_bisection_table (opacityFieldBinding.inl:433-478). */
int gf_field_seal_table(gf_field* field, int64_t token, void* stream);
/* evaluate_bisection_round (opacityFieldBinding.inl:480-521): rounds run in
 * order 0..7 over Q points; above = observed and no camera below 1/2, exact =
 * above and the minimum equals 1/2 exactly; all [Q] uint8.  Synchronizes the
 * stream once, as the reference does. */
int gf_field_evaluate_round(gf_field* field, int64_t token, const float* points, uint32_t num_points,
                            uint32_t round, uint8_t* above, uint8_t* observed, uint8_t* exact, void* stream);
/* reset_bisection_batch (opacityFieldBinding.inl:523-531): after round 7. */
int gf_field_reset_batch(gf_field* field, int64_t token, void* stream);
/* release_bisection_table (opacityFieldBinding.inl:533-545): after round 7. */
int gf_field_release_table(gf_field* field, int64_t token, void* stream);
/* Counters of work done (synchronizes the device).  No reference
 * counterpart (bench accounting). */
int gf_field_get_stats(gf_field* field, gf_field_stats* stats);
/* Per-stage CUDA-event timing of later calls.  No reference counterpart. */
int gf_field_enable_timing(gf_field* field, int enable);
/* Milliseconds and launch counts per GF_FIELD_STAGE_* since the last collect
 * (arrays of GF_FIELD_STAGES; synchronizes the recorded events). */
int gf_field_collect_times(gf_field* field, float* ms, uint32_t* launches);

/* ------------------------------------------------------------------------
 * Physical-mip 3-D filter search.  Replaces best_rate of the reference's
 * gofish_physical_mip extension (threedgrut/physical_mip_csrc/bindings.cpp:
 * 34-101, fused_refresh_cuda.cu:40-219).  For each point [N,3] (float64): the
 * finest pixel sampling rate over the frames whose calibrated support holds
 * its projection (best_rate [N] float64, 0 when none), the winning frame's
 * index (owner [N] int32, -1 when none; equal rates go to the smaller
 * frame_rank), observed [N] uint8, and the unit direction from the winner's
 * centre (direction [N,3] float64, 0 when none).  Frame table: rotations
 * [F,3,3] camera-to-world, centers [F,3], frame_camera / frame_index [F]
 * int32, frame_rank [F] int64.  Camera table (C <= 64): camera_model
 * (threedgrut/physical_mip.py:37-45 ids), width, height [C] int32,
 * camera_params [C,12] float64 as [fx, fy, cx, cy, distortion...],
 * camera_max_angle [C] float64 (-1: none), row_lo / row_hi [C,row_stride]
 * int32 valid column runs per raster row.  All device memory. */
int gf_mip_best_rate(const double* positions, int64_t num_points, const double* rotations, const double* centers,
                     const int32_t* frame_camera, const int32_t* frame_index, const int64_t* frame_rank,
                     int64_t num_frames, const int32_t* camera_model, const int32_t* camera_width,
                     const int32_t* camera_height, const double* camera_params, const double* camera_max_angle,
                     int32_t num_cameras, const int32_t* row_lo, const int32_t* row_hi, int64_t row_stride,
                     double* best_rate, int32_t* owner, uint8_t* observed, double* direction, void* stream);

/* ------------------------------------------------------------------------
 * Per-view full-shape operator (replaces view_observation_filter.
 * current_view_q6, threedgut_tracer/view_observation_filter.py:232-330, the
 * native footprint full-shape operator, footprint_shape_operator.py:51-228 /
 * src/footprint_shape_operator_cuda.cu, and the fused inference kernel
 * src/fast_shape.cu).  All arrays are device memory; float64 arithmetic.
 * ------------------------------------------------------------------------ */

/* The active camera of one view: camera-to-world pose (row-major 4x4), and
 * either OPENCV_FISHEYE (focal, k1..k4, max_angle) or an ideal pinhole
 * (focal only). */
typedef struct gf_shape_camera {
    float c2w[16];
    int32_t fisheye;
    int32_t reserved0;
    float focal_length[2];
    float radial[4];
    float max_angle;
    float reserved1;
} gf_shape_camera;

/* current_view_q6: q6 [N,6] float64 (upper triangle of Q = gamma J^+ J^+^T,
 * order xx xy xz yy yz zz), jacobian [N,2,3] float32 (zero where not
 * observed), observed [N] uint8. */
int gf_view_q6(const float* positions, int64_t n, const gf_shape_camera* camera, double gamma, double* q6,
               float* jacobian, uint8_t* observed, void* stream);

/* Full shape of every row: covariance C = R S^2 R^T + Q, factor B,
 * inverse_factor B^-1 (all [N,3,3] float32), compensation m [N] and
 * out_density [N] (m * density when mass_preserving).  mode 0: B = C^{1/2} R
 * (symmetric root, the training operator); mode 1: B = chol(C).  Unobserved
 * rows: B = R S, m = 1.  status (device, 4 int32): flags in status[0]
 * (1 not positive definite, 2 degenerate projected covariance, 4 non-finite
 * output), the first failing row as uint64 in status[2..3]; reset by the call. */
int gf_full_shape(const float* scales, const float* quaternions, const float* density, const double* q6,
                  const float* jacobian, const uint8_t* observed, int64_t n, double gamma, int mass_preserving,
                  int mode, float* covariance, float* factor, float* inverse_factor, float* compensation,
                  float* out_density, int32_t* status, void* stream);

/* VJP of gf_full_shape (mode 0) to scales [N,3], quaternions [N,4] and
 * density [N]; any output gradient may be NULL (zero). */
int gf_full_shape_bwd(const float* scales, const float* quaternions, const float* density, const double* q6,
                      const float* jacobian, const uint8_t* observed, int64_t n, double gamma, int mass_preserving,
                      const float* grad_covariance, const float* grad_factor, const float* grad_inverse_factor,
                      const float* grad_compensation, const float* grad_density, float* grad_scales,
                      float* grad_quaternions, float* grad_density_in, void* stream);

/* One inference frame: Q, the full shape and m of every row written into the
 * packed [N,32] rows (density slot 3, B 12-20, B^-1 21-29).  mode 0 exact,
 * mode 1 Cholesky with the stored shape for rows whose factorization fails
 * (fast_shape.cu:136-197).  status as for gf_full_shape. */
int gf_view_shape_packed(const float* positions, const float* quaternions, const float* scales,
                         const float* density, int64_t n, const gf_shape_camera* camera, double gamma, int mode,
                         float* packed, int32_t* status, void* stream);

/* The training renderer's packed [N,32] particle rows from the model's
 * per-slot tensors: position [N,3], view density [N], rotation [N,4],
 * intrinsic scale [N,3], intrinsic density [N], factor B [N,9] and B^-1
 * [N,9], padding words zero.  Replaces the torch.concat of
 * threedgut_tracer/tracer.py:171-179.  rows must be 16-byte aligned. */
int gf_pack_particle_rows(const float* positions, const float* density, const float* rotations,
                          const float* scales, const float* intrinsic_density, const float* factor,
                          const float* inverse_factor, int64_t n, float* rows, void* stream);

/* The [N,32] row gradient split back into the per-slot gradients (same
 * layout as gf_pack_particle_rows; padding dropped).  Replaces the
 * torch.split of threedgut_tracer/tracer.py:334-343. */
int gf_unpack_particle_rows(const float* rows, int64_t n, float* positions, float* density, float* rotations,
                            float* scales, float* intrinsic_density, float* factor, float* inverse_factor,
                            void* stream);

/* Tetrahedralization sites of the mesh extraction (gofish/mesh/sites.py:43-83,
 * generate_sites, host numpy in the reference): for every Gaussian with
 * density > 1/255, in order, its centre then the eight corners mu + B (r s)
 * of its support box (s in {-1,+1}^3, x slowest), r = min(sqrt(-2 ln
 * 0.0113f), sqrt(2 ln(255 o))).  Device inputs: positions [N,3], factor B
 * [N,3,3] row-major, density [N], sigma_max [N] (float32).  Device outputs,
 * sized for 9 N sites: points [9N,3] float32, scale [9N] float32 (sigma_max
 * r), owner [9N] int64, *count = kept Gaussians (sites = 9 * count), *status =
 * 1 when a kept Gaussian's radius is not finite and positive.  Scratch is
 * allocated and freed on the stream. */
int gf_mesh_sites(const float* positions, const float* factor, const float* density, const float* sigma_max,
                  uint32_t num_gaussians, float* points, float* scale, int64_t* owner, uint32_t* count,
                  uint32_t* status, void* stream);

/* Marching tetrahedra of the mesh extraction (gofish/mesh/marching_tetrahedra.py:
 * 47-162, marching_tetrahedra on one grid): the crossing edges of the zero
 * level set of sdf (inside: sdf > 0) over tetrahedra tets [T,4] (int64 vertex
 * ids) of vertices [V,3], in the reference's order (distinct edges sorted by
 * (min, max)), and the faces over them (one-triangle tetrahedra, then
 * two-triangle ones, per chunk of the reference's chunking; chunk_tets = 0
 * selects its 32 Mi).  gf_mesh_mt_run classifies, sorts and numbers (two host
 * reads) and returns the edge and face counts; gf_mesh_mt_outputs writes
 * endpoints [E,2,3], endpoint fields [E,2], endpoint scales [E,2] (float32),
 * faces [F,3] and edges [E,2] (int64).  The inputs must stay valid until the
 * outputs are written. */
typedef struct gf_mesh_mt gf_mesh_mt;
gf_mesh_mt* gf_mesh_mt_create(void);
void gf_mesh_mt_destroy(gf_mesh_mt* mt);
int gf_mesh_mt_run(gf_mesh_mt* mt, const float* vertices, uint64_t num_vertices, const int64_t* tets,
                   uint64_t num_tets, const float* sdf, const float* scales, uint64_t chunk_tets,
                   uint64_t* num_edges, uint64_t* num_faces, void* stream);
int gf_mesh_mt_outputs(gf_mesh_mt* mt, float* endpoints, float* endpoint_fields, float* endpoint_scales,
                       int64_t* faces, int64_t* edges, void* stream);

/* SOF's vertex filter (gofish/mesh/filters.py:15-29): keep[e] = 1 when
 * |p_a - p_b| <= scale_a + scale_b for crossing edge e = (a, b). */
int gf_mesh_sof_vertex_filter(const float* points, const float* scale, const int64_t* edges, uint64_t num_edges,
                              uint8_t* keep, void* stream);

/* GOF's cell filter (gofish/mesh/filters.py:42-58): keep[t] = 0 when an edge
 * of tetrahedron t joins two different owners farther apart than the sum of
 * their scales. */
int gf_mesh_gof_cell_filter(const int64_t* cells, uint64_t num_cells, const float* points, const float* scale,
                            const int64_t* owner, uint8_t* keep, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GOFISH_B200_H */
