// Golden-vector generator for the per-hit forward and backward of the
// tracer: runs the reference's own device functions on the host cores.
// Test infrastructure only (built by `make -C oracle ref REF=<reference
// checkout>` into oracle/_ref/, run by tests/golden/make_hit_golden.py).
//
// It includes, unmodified, the reference headers
//   threedgut_tracer/include/3dgut/kernels/cuda/sensors/cameraProjections.cuh
//   (projectPoint, with sensors.h and cameraModels.h over the vector types of
//   tiny-cuda-nn/vec.h here)
//   threedgut_tracer/include/3dgut/kernels/cuda/renderers/gutKBufferRenderer.cuh
//   (HitParticleKBufferT :118-166; its kernel templates are parsed, not used)
//   threedgut_tracer/include/3dgut/kernels/cuda/models/gaussianParticles.cuh
//   (processHitFwd :611-686, processHitBwd :736-1155,
//    particleExactDepthCrossingRaw :592-609,
//    particleAlongRaySigmaIntrinsicPhysicalMip :175-179)
// and the headers they include, compiled with g++ against
// cuda_host_shim.h, with the reference build's defines for the default
// training configuration (configs/render/3dgut.yaml: kernel degree 2,
// min response 0.0113, min alpha 1/255, max alpha 0.99, min transmittance
// 1e-4; setup_3dgut.py:183-191).
//
// Each ray composites one tile's particle list in list order (the K = 0
// order of gutKBufferRenderer.cuh, one candidate after another, stopping
// once the transmittance falls below the minimum), as the renderer's
// per-hit calls do:
//  * forward A: processHitFwd with per-particle (non per-ray) radiance, the
//    colour clamped at zero as the renderer passes it
//    (gutKBufferRenderer.cuh:264-268, :404-405);
//  * forward B: the training channels, accumulated by a walk of
//    processHitBwd with zero output gradients (that walk maintains the same
//    front-to-back sums as the forward: radiance, transmittance, hit
//    distance, sum w t^2, the GOF normal, the intrinsic extent and the
//    clipped inverse-depth moments), plus, from the hit distance of
//    gutHalfRayClosestPoint and the transmittance after each hit, the first
//    depths where the opacity reaches 0.05 ... 0.50 and the exact 0.5
//    crossing with its rate (gutKBufferRenderer.cuh:361-390);
//  * backward: a second walk of processHitBwd with the integrated values of
//    forward B and the given output gradients, the per-hit particle and
//    colour gradients summed per particle
//    (initializeBackwardRay, rayPayloadBackward.cuh:55-139:
//    transmittance gradient = -dL/d(opacity), crossing gradient =
//    -dL/dt* / rate when |rate| > 1e-8 and t* > 0).
//
// Per-hit mode input file (little-endian): int32 tiles, int32 rays_per_tile; per tile
// int32 count then count x float32[32] packed rows and count x float32[3]
// colours; per ray float32[8] (origin, unit direction, t_min, t_max) and
// float32[12] output gradients (rgb, opacity, hit distance, normal xyz,
// sum w t^2, extent, inverse depth, inverse depth squared) and float32 dL/dt*.
// Output file: per ray float32[6] forward A (rgb, opacity, hit distance,
// hit count), float32[19] forward B (rgb, opacity, hit distance, normal xyz,
// sum w t^2, extent, inverse depth, inverse depth squared, seven quantile
// depths) + float32[2] (exact crossing depth, its rate); per tile and
// particle float32[32] particle gradient (ParticleDensity layout),
// float32[3] colour gradient and float32[3] sum over its hits of the absolute
// values of the hit's position gradient (the world-space densification
// statistic).

#include "cuda_host_shim.h"

#include <3dgut/kernels/cuda/models/gaussianParticles.cuh>
#include <3dgut/kernels/cuda/sensors/cameraProjections.cuh>
#include <3dgut/kernels/cuda/renderers/gutKBufferRenderer.cuh>

// The projector's compile-time configuration, which the reference's
// threedgut.cuh:56-69 builds from the build defines before it includes
// gutProjector.cuh; the UT projection reads ParticleMinSensorZ and
// AlphaThreshold, the other members only have to exist.
struct TGUTProjectorParams {
    static constexpr float ParticleMinSensorZ = threedgut::kParticleMinSensorZ;
    static constexpr float CovarianceDilation = 0.3f;
    static constexpr float AlphaThreshold = GAUSSIAN_PARTICLE_MIN_ALPHA;
    static constexpr bool TightOpacityBounding = true;
    static constexpr bool RectBounding = true;
    static constexpr bool TileCulling = true;
    static constexpr bool PerRayParticleFeatures = false;
    static constexpr float MaxDepthValue = 3.4028235e+38f;
    static constexpr bool GlobalZOrder = false;
    static constexpr bool PerTileDepth = true;
    static constexpr bool BackwardProjection = false;
    static constexpr bool MipSplattingScaling = true;
};
#include <3dgut/kernels/cuda/renderers/gutProjector.cuh>

#include <cstdio>
#include <cstdlib>
#include <vector>

namespace {

constexpr float kMinResponse = GAUSSIAN_PARTICLE_MIN_KERNEL_DENSITY;
constexpr float kMinAlpha = GAUSSIAN_PARTICLE_MIN_ALPHA;
constexpr float kMinTransmittance = GAUSSIAN_MIN_TRANSMITTANCE_THRESHOLD;
constexpr int kKernelDegree = GAUSSIAN_PARTICLE_KERNEL_DEGREE;
constexpr int kQuantiles = 7;
constexpr float kQuantileLevels[kQuantiles] = {0.05f, 0.10f, 0.15f, 0.20f, 0.30f, 0.40f, 0.50f};

static_assert(sizeof(threedgut::ParticleDensity) == 32 * sizeof(float), "packed particle row is 32 floats");

struct Ray {
    float3 o, d;
    float tmin, tmax;
};

struct Accum {
    float T = 1.0f;
    float3 rgb = make_float3(0.0f, 0.0f, 0.0f);
    float depth = 0.0f;
    float sumWD2 = 0.0f;
    float3 normal = make_float3(0.0f, 0.0f, 0.0f);
    float sumExt = 0.0f;
    float sumWinvD = 0.0f;
    float sumWinvD2 = 0.0f;
};

bool read_all(FILE* f, void* p, size_t bytes) { return fread(p, 1, bytes, f) == bytes; }

}  // namespace

// `sh` mode: the particle radiance of the projector,
// radianceFromSpH(degree, coefficients, incident direction, unclamped)
// (gaussianParticles.cuh:188-220 as gutProjector.cuh:903 calls it).  Input:
// int32 count, int32 degree, then per item float32[3] unit direction and
// float32[48] coefficients (16 x rgb); output per item float32[3].
int run_sh(const char* inPath, const char* outPath) {
    FILE* in = fopen(inPath, "rb");
    if (in == nullptr) return 3;
    int32_t count = 0, degree = 0;
    if (!read_all(in, &count, 4) || !read_all(in, &degree, 4)) return 4;
    FILE* out = fopen(outPath, "wb");
    if (out == nullptr) return 5;
    for (int i = 0; i < count; ++i) {
        float3 dir;
        float3 coeffs[16];
        if (!read_all(in, &dir, sizeof(dir)) || !read_all(in, coeffs, sizeof(coeffs))) return 6;
        const float3 rgb = threedgut::radianceFromSpH(degree, coeffs, dir, false);
        fwrite(&rgb, sizeof(float3), 1, out);
    }
    fclose(out);
    fclose(in);
    return 0;
}

// `project` mode: the sensor-space point projection of the UT sigma points,
// projectPoint of cameraProjections.cuh:75-122 (OpenCV pinhole) and :124-152
// (OpenCV fisheye / Kannala-Brandt) with requireRasterBounds = false, as
// gutProjector.cuh calls it.  Input: int32 count, int32 model (0 pinhole, 1
// fisheye), int32 width, int32 height, float32 principal[2], focal[2],
// radial[6], tangential[2], thin_prism[4], max_angle, tolerance, then per point
// float32[3]; output per point float32 u, v, valid (0 or 1).
int run_project(const char* inPath, const char* outPath) {
    FILE* in = fopen(inPath, "rb");
    if (in == nullptr) return 3;
    int32_t head[4];
    float cam[18];
    if (!read_all(in, head, sizeof(head)) || !read_all(in, cam, sizeof(cam))) return 4;
    FILE* out = fopen(outPath, "wb");
    if (out == nullptr) return 5;
    threedgut::OpenCVPinholeProjectionParameters pin{};
    threedgut::OpenCVFisheyeProjectionParameters fish{};
    pin.principalPoint = tcnn::vec2(cam[0], cam[1]);
    pin.focalLength = tcnn::vec2(cam[2], cam[3]);
    for (int i = 0; i < 6; ++i) pin.radialCoeffs[i] = cam[4 + i];
    pin.tangentialCoeffs = tcnn::vec2(cam[10], cam[11]);
    pin.thinPrismCoeffs = tcnn::vec4(cam[12], cam[13], cam[14], cam[15]);
    fish.principalPoint = pin.principalPoint;
    fish.focalLength = pin.focalLength;
    for (int i = 0; i < 4; ++i) fish.radialCoeffs[i] = cam[4 + i];
    fish.maxAngle = cam[16];
    const tcnn::ivec2 resolution(head[2], head[3]);
    for (int i = 0; i < head[0]; ++i) {
        float p[3];
        if (!read_all(in, p, sizeof(p))) return 6;
        tcnn::vec2 uv;
        const tcnn::vec3 position(p[0], p[1], p[2]);
        const bool valid = head[1] == 1 ? threedgut::projectPoint(fish, resolution, position, cam[17], uv, false)
                                        : threedgut::projectPoint(pin, resolution, position, cam[17], uv, false);
        const float rec[3] = {uv.x, uv.y, valid ? 1.0f : 0.0f};
        fwrite(rec, sizeof(float), 3, out);
    }
    fclose(out);
    fclose(in);
    return 0;
}

// `kbuffer` mode: the composite order of the k-buffer, the reference's
// HitParticleKBufferT<K>::insert (gutKBufferRenderer.cuh:118-166) fed as
// evalKBuffer feeds it (:676-699: when full, composite the closest entry,
// then insert; at the end composite the held entries from the closest).
// Input: int32 sequences, then per sequence int32 K, int32 n and n float32 hit
// distances (hit i has id i); output per sequence the n ids in composite order.
template <int K>
void kbuffer_order(const float* hitT, int n, int32_t* order) {
    ::HitParticleKBufferT<K, false> kb;
    int at = 0;
    for (int i = 0; i < n; ++i) {
        ::HitParticleT<false> h;
        h.idx = i;
        h.hitT = hitT[i];
        h.alpha = 0.5f;
        if (kb.full()) order[at++] = kb.closestHit(h).idx;
        kb.insert(h);
    }
    for (uint32_t i = 0; i < kb.numHits(); ++i) order[at++] = kb[K - kb.numHits() + i].idx;
}

int run_kbuffer(const char* inPath, const char* outPath) {
    FILE* in = fopen(inPath, "rb");
    if (in == nullptr) return 3;
    int32_t sequences = 0;
    if (!read_all(in, &sequences, 4)) return 4;
    FILE* out = fopen(outPath, "wb");
    if (out == nullptr) return 5;
    for (int sq = 0; sq < sequences; ++sq) {
        int32_t head[2];
        if (!read_all(in, head, sizeof(head))) return 6;
        std::vector<float> hitT(static_cast<size_t>(head[1]));
        std::vector<int32_t> order(static_cast<size_t>(head[1]), -1);
        if (!read_all(in, hitT.data(), sizeof(float) * hitT.size())) return 7;
        switch (head[0]) {
            case 4: kbuffer_order<4>(hitT.data(), head[1], order.data()); break;
            case 8: kbuffer_order<8>(hitT.data(), head[1], order.data()); break;
            case 12: kbuffer_order<12>(hitT.data(), head[1], order.data()); break;
            case 16: kbuffer_order<16>(hitT.data(), head[1], order.data()); break;
            case 24: kbuffer_order<24>(hitT.data(), head[1], order.data()); break;
            case 32: kbuffer_order<32>(hitT.data(), head[1], order.data()); break;
            default: return 8;
        }
        fwrite(order.data(), sizeof(int32_t), order.size(), out);
    }
    fclose(out);
    fclose(in);
    return 0;
}

// `ut` mode: GUTProjector::unscentedParticleProjection (gutProjector.cuh:359-518),
// the 7-point unscented transform of a particle through a global-shutter
// camera, with the reference's default UT parameters
// (threedgut.cuh:72-81 with configs/render/3dgut.yaml: alpha 1, beta 2,
// kappa 0, delta sqrt(3), 10% image margin, not every sigma point required).
// The particle model is reached through three accessors, restated here as
// the reference's shRadiativeGaussianParticles.cuh:89-123 defines them (the
// model class itself is built from Slang-generated code): position = slots
// 0-2, opacity = slot 3, factorColumn(i) = column i of the row-major B in
// slots 12-20.
struct UtParams {
    static constexpr int NRollingShutterIterations = 1;
    static constexpr int D = 3;
    static constexpr float Alpha = 1.0f;
    static constexpr float Beta = 2.0f;
    static constexpr float Kappa = 0.0f;
    static constexpr float Delta = 1.7320508075688772f;
    static constexpr float ImageMarginFactor = 0.1f;
    static constexpr bool RequireAllSigmaPoints = false;
};

struct PackedRowParticles {
    using DensityParameters = threedgut::ParticleDensity;
    using TFeaturesVec = tcnn::vec3;  // named by the projector's declarations only
    const tcnn::vec3& position(const DensityParameters& p) const {
        return *reinterpret_cast<const tcnn::vec3*>(&p.position);
    }
    const float& opacity(const DensityParameters& p) const { return p.density; }
    tcnn::vec3 factorColumn(const DensityParameters& p, int axis) const {
        const float* b = &p.factor[0].x;
        return tcnn::vec3(b[axis], b[3 + axis], b[6 + axis]);
    }
};

// Input: int32 count, int32 model, int32 width, int32 height, float32
// camera[18] (as `project`), float32 pose[7] (world->sensor t, q xyzw),
// float32 centre[3] (the sensor position in the world), then count packed
// rows; output per particle float32 centre u, v, covariance xx, xy, yy, valid.
int run_ut(const char* inPath, const char* outPath) {
    using Projector = GUTProjector<PackedRowParticles, TGUTProjectorParams, UtParams>;
    FILE* in = fopen(inPath, "rb");
    if (in == nullptr) return 3;
    int32_t head[4];
    float cam[18], pose[7], centre[3];
    if (!read_all(in, head, sizeof(head)) || !read_all(in, cam, sizeof(cam)) || !read_all(in, pose, sizeof(pose)) ||
        !read_all(in, centre, sizeof(centre)))
        return 4;
    FILE* out = fopen(outPath, "wb");
    if (out == nullptr) return 5;
    threedgut::TSensorModel model{};
    model.shutterType = threedgut::TSensorModel::GlobalShutter;
    if (head[1] == 1) {
        model.modelType = threedgut::TSensorModel::OpenCVFisheyeModel;
        model.ocvFisheyeParams.principalPoint = tcnn::vec2(cam[0], cam[1]);
        model.ocvFisheyeParams.focalLength = tcnn::vec2(cam[2], cam[3]);
        for (int i = 0; i < 4; ++i) model.ocvFisheyeParams.radialCoeffs[i] = cam[4 + i];
        model.ocvFisheyeParams.maxAngle = cam[16];
    } else {
        model.modelType = threedgut::TSensorModel::OpenCVPinholeModel;
        model.ocvPinholeParams.principalPoint = tcnn::vec2(cam[0], cam[1]);
        model.ocvPinholeParams.focalLength = tcnn::vec2(cam[2], cam[3]);
        for (int i = 0; i < 6; ++i) model.ocvPinholeParams.radialCoeffs[i] = cam[4 + i];
        model.ocvPinholeParams.tangentialCoeffs = tcnn::vec2(cam[10], cam[11]);
        model.ocvPinholeParams.thinPrismCoeffs = tcnn::vec4(cam[12], cam[13], cam[14], cam[15]);
    }
    threedgut::TSensorState state{};
    for (int i = 0; i < 7; ++i) state.startPose[i] = state.endPose[i] = pose[i];
    state.startTimestamp = 0;
    state.endTimestamp = 1;
    const tcnn::mat4x3 sensorMatrix = threedgut::sensorPoseToMat(state.startPose);
    const tcnn::vec3 sensorPosition(centre[0], centre[1], centre[2]);
    const tcnn::ivec2 resolution(head[2], head[3]);
    PackedRowParticles particles;
    for (int i = 0; i < head[0]; ++i) {
        threedgut::ParticleDensity row;
        if (!read_all(in, &row, sizeof(row))) return 6;
        tcnn::vec3 sensorRay, cov(0.0f);
        tcnn::vec2 centreUv(0.0f);
        float opacity = 0.0f;
        bool capEligible = false;
        const bool valid = Projector::unscentedParticleProjection(resolution, model, sensorPosition, sensorMatrix, state,
                                                                  particles, row, sensorRay, opacity, centreUv, cov,
                                                                  capEligible);
        const float rec[6] = {centreUv.x, centreUv.y, cov.x, cov.y, cov.z, valid ? 1.0f : 0.0f};
        fwrite(rec, sizeof(float), 6, out);
    }
    fclose(out);
    fclose(in);
    return 0;
}

int main(int argc, char** argv) {
    if (argc == 4 && strcmp(argv[1], "ut") == 0) return run_ut(argv[2], argv[3]);
    if (argc == 4 && strcmp(argv[1], "kbuffer") == 0) return run_kbuffer(argv[2], argv[3]);
    if (argc == 4 && strcmp(argv[1], "sh") == 0) return run_sh(argv[2], argv[3]);
    if (argc == 4 && strcmp(argv[1], "project") == 0) return run_project(argv[2], argv[3]);
    if (argc != 3) {
        fprintf(stderr, "usage: %s input.bin output.bin | %s sh input.bin output.bin\n", argv[0], argv[0]);
        return 2;
    }
    FILE* in = fopen(argv[1], "rb");
    if (in == nullptr) return 3;
    int32_t tiles = 0, raysPerTile = 0;
    if (!read_all(in, &tiles, 4) || !read_all(in, &raysPerTile, 4)) return 4;
    FILE* out = fopen(argv[2], "wb");
    if (out == nullptr) return 5;

    for (int tile = 0; tile < tiles; ++tile) {
        int32_t count = 0;
        if (!read_all(in, &count, 4)) return 6;
        std::vector<threedgut::ParticleDensity> particles(static_cast<size_t>(count));
        std::vector<float3> colours(static_cast<size_t>(count));
        if (!read_all(in, particles.data(), sizeof(threedgut::ParticleDensity) * size_t(count))) return 7;
        if (!read_all(in, colours.data(), sizeof(float3) * size_t(count))) return 8;
        for (auto& c : colours) c = make_float3(fmaxf(c.x, 0.0f), fmaxf(c.y, 0.0f), fmaxf(c.z, 0.0f));
        std::vector<threedgut::ParticleDensity> gradSum(static_cast<size_t>(count));
        std::vector<float3> colourGradSum(size_t(count), make_float3(0.0f, 0.0f, 0.0f));
        std::vector<float3> absSum(size_t(count), make_float3(0.0f, 0.0f, 0.0f));
        memset(gradSum.data(), 0, sizeof(threedgut::ParticleDensity) * size_t(count));

        for (int r = 0; r < raysPerTile; ++r) {
            float rayIn[8], gradIn[12], dLdtStar = 0.0f;
            if (!read_all(in, rayIn, sizeof(rayIn)) || !read_all(in, gradIn, sizeof(gradIn)) ||
                !read_all(in, &dLdtStar, 4))
                return 9;
            const Ray ray{make_float3(rayIn[0], rayIn[1], rayIn[2]), make_float3(rayIn[3], rayIn[4], rayIn[5]),
                          rayIn[6], rayIn[7]};

            // forward A: processHitFwd
            float fT = 1.0f, fDepth = 0.0f;
            float3 fRgb = make_float3(0.0f, 0.0f, 0.0f);
            float hits = 0.0f;
            for (int i = 0; i < count && fT >= kMinTransmittance; ++i) {
                const bool hit = threedgut::processHitFwd<kKernelDegree, false, false>(
                    ray.o, ray.d, i, particles.data(), reinterpret_cast<const float*>(colours.data()), kMinResponse,
                    kMinAlpha, 0, &fT, &fRgb, &fDepth, nullptr, ray.tmin, ray.tmax);
                if (hit) hits += 1.0f;
            }

            // forward B: processHitBwd walk with zero output gradients
            Accum acc;
            float quant[kQuantiles] = {};
            float exactDepth = 0.0f, exactRate = 0.0f;
            for (int i = 0; i < count && acc.T >= kMinTransmittance; ++i) {
                threedgut::ParticleDensity scratch;
                memset(&scratch, 0, sizeof(scratch));
                float colourGrad[3] = {};
                const float before = acc.T;
                threedgut::processHitBwd<kKernelDegree, false, false>(
                    ray.o, ray.d, uint32_t(i), particles[size_t(i)], &scratch,
                    reinterpret_cast<const float*>(&colours[size_t(i)]), colourGrad, kMinResponse, kMinAlpha,
                    kMinTransmittance, 0, 0.0f, acc.T, 0.0f, make_float3(0.0f, 0.0f, 0.0f), acc.rgb,
                    make_float3(0.0f, 0.0f, 0.0f), 0.0f, acc.depth, 0.0f, 0.0f, &acc.sumWD2, 0.0f, &acc.normal,
                    make_float3(0.0f, 0.0f, 0.0f), make_float3(0.0f, 0.0f, 0.0f), 0.0f, &acc.sumExt, 0.0f, 0.0f,
                    0.0f, 0.0f, 0.0f, &acc.sumWinvD, 0.0f, 0.0f, &acc.sumWinvD2, 0.0f, 0.0f, 0.0f, ray.tmin,
                    ray.tmax, 1.0f);
                if (acc.T != before) {
                    // the hit distance of the accepted hit (gutHalfRayResponse.cuh:17-37)
                    float hitT = 0.0f;
                    threedgut::intersectCustomParticle(ray.o, ray.d, i, particles.data(), ray.tmin, ray.tmax,
                                                       1e30f, hitT);
                    const float opacity = 1.0f - acc.T;
                    for (int q = 0; q < kQuantiles; ++q)
                        if (quant[q] == 0.0f && opacity >= kQuantileLevels[q]) quant[q] = hitT;
                    if (exactDepth == 0.0f && before > 0.5f && acc.T <= 0.5f) {
                        const threedgut::FiniteIntervalCrossingResult c = threedgut::particleExactDepthCrossingRaw(
                            particles[size_t(i)], ray.o, ray.d, before, ray.tmin, ray.tmax);
                        exactDepth = c.valid ? c.depth : hitT;
                        exactRate = c.valid ? c.rate : 0.0f;
                    }
                }
            }

            // backward: processHitBwd walk with the integrated values of forward B
            const float3 gRgb = make_float3(gradIn[0], gradIn[1], gradIn[2]);
            const float gT = -1.0f * gradIn[3];
            const float3 gNormal = make_float3(gradIn[5], gradIn[6], gradIn[7]);
            const float crossingGrad = (fabsf(exactRate) > 1e-8f && exactDepth > 0.0f) ? (-dLdtStar / exactRate)
                                                                                       : 0.0f;
            Accum run;
            for (int i = 0; i < count && run.T >= kMinTransmittance; ++i) {
                threedgut::ParticleDensity g;
                memset(&g, 0, sizeof(g));
                float colourGrad[3] = {};
                threedgut::processHitBwd<kKernelDegree, false, false>(
                    ray.o, ray.d, uint32_t(i), particles[size_t(i)], &g,
                    reinterpret_cast<const float*>(&colours[size_t(i)]), colourGrad, kMinResponse, kMinAlpha,
                    kMinTransmittance, 0, acc.T, run.T, gT, acc.rgb, run.rgb, gRgb, acc.depth, run.depth, gradIn[4],
                    acc.sumWD2, &run.sumWD2, gradIn[8], &run.normal, acc.normal, gNormal, acc.sumExt, &run.sumExt,
                    gradIn[9], 0.0f, 0.0f, 0.0f, acc.sumWinvD, &run.sumWinvD, gradIn[10], acc.sumWinvD2,
                    &run.sumWinvD2, gradIn[11], crossingGrad, exactDepth, ray.tmin, ray.tmax, 1.0f);
                float* dst = reinterpret_cast<float*>(&gradSum[size_t(i)]);
                const float* src = reinterpret_cast<const float*>(&g);
                for (int k = 0; k < 32; ++k) dst[k] += src[k];
                // the world-space densification statistic (gutKBufferRenderer.cuh:290-294)
                absSum[size_t(i)].x += fabsf(g.position.x);
                absSum[size_t(i)].y += fabsf(g.position.y);
                absSum[size_t(i)].z += fabsf(g.position.z);
                colourGradSum[size_t(i)].x += colourGrad[0];
                colourGradSum[size_t(i)].y += colourGrad[1];
                colourGradSum[size_t(i)].z += colourGrad[2];
            }

            const float fwdA[6] = {fRgb.x, fRgb.y, fRgb.z, 1.0f - fT, fDepth, hits};
            const float fwdB[21] = {acc.rgb.x, acc.rgb.y, acc.rgb.z, 1.0f - acc.T, acc.depth, acc.normal.x,
                                    acc.normal.y, acc.normal.z, acc.sumWD2, acc.sumExt, acc.sumWinvD, acc.sumWinvD2,
                                    quant[0], quant[1], quant[2], quant[3], quant[4], quant[5], quant[6],
                                    exactDepth, exactRate};
            fwrite(fwdA, sizeof(float), 6, out);
            fwrite(fwdB, sizeof(float), 21, out);
        }
        fwrite(gradSum.data(), sizeof(threedgut::ParticleDensity), size_t(count), out);
        fwrite(colourGradSum.data(), sizeof(float3), size_t(count), out);
        fwrite(absSum.data(), sizeof(float3), size_t(count), out);
    }
    fclose(out);
    fclose(in);
    return 0;
}
