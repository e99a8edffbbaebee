/*
 * CPU oracle for the Gaussian-splat rasterizer -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's rasterizer kernels
 * (VikaasVarma/gaussian-splats, src/gaussian_splats/kernels/rasterize/):
 *   gso_project       project.py:10-253       (_evaluate_sh, _project_and_count_kernel)
 *   gso_bin           intersections.py:10-88  (emit, stable key sort, tile ranges)
 *   gso_composite     composite.py:25-107     (front-to-back compositing)
 *   gso_composite_bwd composite_bwd.py:47-277 (reverse compositing, per-intersection
 *                                              rows reduced per Gaussian like index_add_)
 *   gso_project_bwd   project_bwd.py:8-334    (parameter VJPs)
 *   gso_adam_step     training/train.py:118,151 + training/utils.py:50-62
 *                                             (torch Adam step, position noise)
 *   gso_relocate      training/utils.py:94-101,120-145,187-193
 *                                             (copy_splats with normalize_copies,
 *                                              moment reset of relocate_splats)
 * Each function follows the reference's float32 operation order (no fused
 * multiply-adds unless written as fmaf) so that integer decisions match the
 * CUDA kernels bit for bit; exp/log come from detmath.h. Only tests, the
 * smoke check and the benchmark's CPU-baseline leg may call this library --
 * it is the checker, never the product path.
 *
 * Deliberate choices where the reference leaves behaviour undefined:
 *  - opacity < 1/255 makes the reference's radius NaN; Triton's clamp then
 *    yields bounds 0 and count 0, which is what happens here;
 *  - the key sort is stable (ties in (tile, depth bits) keep emission order);
 *  - the backward differentiates SH degree 4 too (coefficients 16..24 and
 *    their share of the view-direction gradient), where the reference stops
 *    at 16 and leaves the rest uninitialised (project_bwd.py:33,355);
 *  - ellipsoid rendering has a backward (colour and opacity gradients; the
 *    indicator falloff has none), which the reference refuses
 *    (interface.py:184-186).
 * Pair evaluation inside compositing (shared by forward and backward):
 *    dx = x - mean_x, dy = y - mean_y (integer pixel coordinates, no +0.5)
 *    d2 = fmaf(xx*dx, dx, fmaf((2*xy)*dx, dy, (yy*dy)*dy))
 * which is the reference's xx*dx*dx + 2*xy*dx*dy + yy*dy*dy with two of its
 * roundings fused; colour accumulation is C = fmaf(T*alpha, c, C).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "detmath.h"

#ifdef _OPENMP
#include <omp.h>
#endif

/* Host threads of the parallel loops below. Set explicitly by the benchmark:
 * launchers such as torchrun export OMP_NUM_THREADS=1, which would otherwise
 * leave a timed run on one core while reporting all of them. */
void gso_set_threads(int32_t threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

int32_t gso_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

typedef struct gso_params {
    float fx, fy, cx, cy;
    int32_t width, height, tile_size;
    int32_t gaussian_mode;   /* 1 = gaussian falloff, 0 = ellipsoid indicator */
    float near_plane, far_plane;
    float lim_x, lim_y;      /* 1.3 * W / (2 fx), folded in double by the host (project.py:158-159) */
    float bwd_lim_x, bwd_lim_y; /* same limits as project_bwd.py:376-377 folds them */
    float extent;            /* ellipsoid radius multiplier sqrt(-2 log1p(-confidence)) */
    float cutoff;            /* ellipsoid d^2 cutoff -2 log1p(-confidence) */
    float opacity_threshold;
} gso_params;

#define ALPHA_MIN (1.0f / 255.0f)

/* ---------------------------------------------------------------- project */

static float sh_basis(int k, float x, float y, float z, float xx, float yy, float zz) {
    /* project.py:22-61 (forward constants). */
    switch (k) {
    case 0: return 0.28209479177387814f;
    case 1: return -0.4886025119029199f * y;
    case 2: return 0.4886025119029199f * z;
    case 3: return -0.4886025119029199f * x;
    case 4: return 1.0925484305920792f * x * y;
    case 5: return -1.0925484305920792f * y * z;
    case 6: return 0.31539156525252005f * (2.0f * zz - xx - yy);
    case 7: return -1.0925484305920792f * x * z;
    case 8: return 0.5462742152960396f * (xx - yy);
    case 9: return -0.5900435899266435f * y * (3.0f * xx - yy);
    case 10: return 2.890611442640554f * x * y * z;
    case 11: return -0.4570457994644658f * y * (4.0f * zz - xx - yy);
    case 12: return 0.3731763325901154f * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    case 13: return -0.4570457994644658f * x * (4.0f * zz - xx - yy);
    case 14: return 1.445305721320277f * z * (xx - yy);
    case 15: return -0.5900435899266435f * x * (xx - 3.0f * yy);
    case 16: return 2.5033429417967046f * x * y * (xx - yy);
    case 17: return -1.7701307697799304f * y * z * (3.0f * xx - yy);
    case 18: return 0.9461746957575601f * x * y * (7.0f * zz - 1.0f);
    case 19: return -0.6690465435572892f * y * z * (7.0f * zz - 3.0f);
    case 20: return 0.10578554691520431f * (zz * (35.0f * zz - 30.0f) + 3.0f);
    case 21: return -0.6690465435572892f * x * z * (7.0f * zz - 3.0f);
    case 22: return 0.47308734787878004f * (xx - yy) * (7.0f * zz - 1.0f);
    case 23: return -1.7701307697799304f * x * z * (xx - 3.0f * yy);
    default: return 0.6258357354491761f * (xx * (xx - 3.0f * yy) - yy * (3.0f * xx - yy));
    }
}

static void project_one(int64_t i, const float *mean, const float *rotation, const float *scale,
                        const float *opacity, const float *color, int32_t num_sh, const float *R,
                        const float *t, const gso_params *p, float *projected_mean,
                        float *inverse_covariance, float *projected_color,
                        float *projected_opacity, int32_t *bounds, int32_t *counts) {
    const float cr00 = R[0], cr01 = R[1], cr02 = R[2], cr10 = R[3], cr11 = R[4], cr12 = R[5],
                cr20 = R[6], cr21 = R[7], cr22 = R[8];
    const float tx = t[0], ty = t[1], tz = t[2];
    const float mx = mean[3 * i], my = mean[3 * i + 1], mz = mean[3 * i + 2];
    /* project.py:126-142 */
    float camera_x = mx * cr00 + my * cr01 + mz * cr02 + tx;
    float camera_y = mx * cr10 + my * cr11 + mz * cr12 + ty;
    float camera_z = mx * cr20 + my * cr21 + mz * cr22 + tz;
    float depth = -camera_z;
    float safe_z = depth > 0.0f ? fmaxf(1e-4f, depth) : fminf(-1e-4f, depth);
    float pixel_x = p->fx * camera_x / safe_z + p->cx;
    float pixel_y = -p->fy * camera_y / safe_z + p->cy;
    projected_mean[3 * i] = pixel_x;
    projected_mean[3 * i + 1] = pixel_y;
    projected_mean[3 * i + 2] = safe_z;
    /* project.py:144-156 */
    float qw = rotation[4 * i], qx = rotation[4 * i + 1], qy = rotation[4 * i + 2],
          qz = rotation[4 * i + 3];
    float inverse_norm = gso_rsqrt(qw * qw + qx * qx + qy * qy + qz * qz);
    qw = qw * inverse_norm; qx = qx * inverse_norm; qy = qy * inverse_norm; qz = qz * inverse_norm;
    /* project.py:158-168 */
    float cov_x = fminf(p->lim_x, fmaxf(-p->lim_x, camera_x / safe_z)) * safe_z;
    float cov_y = fminf(p->lim_y, fmaxf(-p->lim_y, camera_y / safe_z)) * safe_z;
    float inverse_z = 1.0f / safe_z;
    float j00 = p->fx * inverse_z;
    float j02 = p->fx * cov_x * inverse_z * inverse_z;
    float j11 = -p->fy * inverse_z;
    float j12 = -p->fy * cov_y * inverse_z * inverse_z;
    /* project.py:169-176 */
    float jc00 = j00 * cr00 + j02 * cr20, jc01 = j00 * cr01 + j02 * cr21,
          jc02 = j00 * cr02 + j02 * cr22;
    float jc10 = j11 * cr10 + j12 * cr20, jc11 = j11 * cr11 + j12 * cr21,
          jc12 = j11 * cr12 + j12 * cr22;
    /* project.py:177-213 */
    float sx = gso_exp(scale[3 * i]), sy = gso_exp(scale[3 * i + 1]), sz = gso_exp(scale[3 * i + 2]);
    float a0x = (1.0f - 2.0f * (qy * qy + qz * qz)) * sx;
    float a0y = (2.0f * (qx * qy + qw * qz)) * sx;
    float a0z = (2.0f * (qx * qz - qw * qy)) * sx;
    float a1x = (2.0f * (qx * qy - qw * qz)) * sy;
    float a1y = (1.0f - 2.0f * (qx * qx + qz * qz)) * sy;
    float a1z = (2.0f * (qy * qz + qw * qx)) * sy;
    float a2x = (2.0f * (qx * qz + qw * qy)) * sz;
    float a2y = (2.0f * (qy * qz - qw * qx)) * sz;
    float a2z = (1.0f - 2.0f * (qx * qx + qy * qy)) * sz;
    float f00 = jc00 * a0x + jc01 * a0y + jc02 * a0z;
    float f01 = jc00 * a1x + jc01 * a1y + jc02 * a1z;
    float f02 = jc00 * a2x + jc01 * a2y + jc02 * a2z;
    float f10 = jc10 * a0x + jc11 * a0y + jc12 * a0z;
    float f11 = jc10 * a1x + jc11 * a1y + jc12 * a1z;
    float f12 = jc10 * a2x + jc11 * a2y + jc12 * a2z;
    float cov00 = f00 * f00 + f01 * f01 + f02 * f02 + 0.03f;
    float cov01 = f00 * f10 + f01 * f11 + f02 * f12;
    float cov11 = f10 * f10 + f11 * f11 + f12 * f12 + 0.03f;
    /* project.py:214-218 */
    float determinant = cov00 * cov11 - cov01 * cov01;
    inverse_covariance[4 * i] = cov11 / determinant;
    inverse_covariance[4 * i + 1] = -cov01 / determinant;
    inverse_covariance[4 * i + 2] = -cov01 / determinant;
    inverse_covariance[4 * i + 3] = cov00 / determinant;
    /* project.py:221-228 and _evaluate_sh (project.py:10-71) */
    float dx = mx + cr00 * tx + cr10 * ty + cr20 * tz;
    float dy = my + cr01 * tx + cr11 * ty + cr21 * tz;
    float dz = mz + cr02 * tx + cr12 * ty + cr22 * tz;
    float direction_norm = gso_rsqrt(dx * dx + dy * dy + dz * dz);
    dx = dx * direction_norm; dy = dy * direction_norm; dz = dz * direction_norm;
    float xx = dx * dx, yy = dy * dy, zz = dz * dz;
    const float *coefficients = color + i * (int64_t)num_sh * 3;
    float acc_r = 0.0f, acc_g = 0.0f, acc_b = 0.0f;
    for (int k = 0; k < num_sh; ++k) {
        float b = sh_basis(k, dx, dy, dz, xx, yy, zz);
        acc_r = fmaf(coefficients[3 * k], b, acc_r);
        acc_g = fmaf(coefficients[3 * k + 1], b, acc_g);
        acc_b = fmaf(coefficients[3 * k + 2], b, acc_b);
    }
    projected_color[3 * i] = fmaxf(acc_r + 0.5f, 0.0f);
    projected_color[3 * i + 1] = fmaxf(acc_g + 0.5f, 0.0f);
    projected_color[3 * i + 2] = fmaxf(acc_b + 0.5f, 0.0f);
    /* project.py:230-253 */
    float o = gso_sigmoid(opacity[i]);
    projected_opacity[i] = o;
    float radius_extent = p->gaussian_mode ? 2.0f * sqrtf(gso_log(o * 255.0f)) : p->extent;
    float radius_x = radius_extent * sqrtf(cov00);
    float radius_y = radius_extent * sqrtf(cov11);
    const float ts = (float)p->tile_size;
    const float tiles_w = (float)(p->width / p->tile_size), tiles_h = (float)(p->height / p->tile_size);
    /* tl.clamp: max then min, a NaN operand yields the other one (bound 0). */
    float tmin_x = fminf(fmaxf(floorf((pixel_x - radius_x) / ts), 0.0f), tiles_w);
    float tmin_y = fminf(fmaxf(floorf((pixel_y - radius_y) / ts), 0.0f), tiles_h);
    float tmax_x = fminf(fmaxf(floorf((pixel_x + radius_x) / ts) + 1.0f, 0.0f), tiles_w);
    float tmax_y = fminf(fmaxf(floorf((pixel_y + radius_y) / ts) + 1.0f, 0.0f), tiles_h);
    bounds[4 * i] = (int32_t)tmin_x;
    bounds[4 * i + 1] = (int32_t)tmax_x;
    bounds[4 * i + 2] = (int32_t)tmin_y;
    bounds[4 * i + 3] = (int32_t)tmax_y;
    float count = (tmax_x - tmin_x) * (tmax_y - tmin_y);
    counts[i] = (safe_z > p->near_plane && safe_z < p->far_plane) ? (int32_t)count : 0;
}

void gso_project(int64_t n, const float *mean, const float *rotation, const float *scale,
                 const float *opacity, const float *color, int32_t num_sh, const float *R,
                 const float *t, const gso_params *p, float *projected_mean,
                 float *inverse_covariance, float *projected_color, float *projected_opacity,
                 int32_t *bounds, int32_t *counts) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        project_one(i, mean, rotation, scale, opacity, color, num_sh, R, t, p, projected_mean,
                    inverse_covariance, projected_color, projected_opacity, bounds, counts);
}

/* ---------------------------------------------------------------- binning */

/* Number of intersections (sum of counts); needed to size gso_bin's outputs. */
int64_t gso_total(int64_t n, const int32_t *counts) {
    int64_t total = 0;
    for (int64_t i = 0; i < n; ++i) total += counts[i];
    return total;
}

/* Emit keys (tile << 32 | depth bits) in Gaussian-major order
 * (intersections.py:10-41), stable-sort them (intersections.py:82-83) and
 * turn per-tile counts into [start, end) ranges (intersections.py:84-88).
 * keys_out/ids_out (may be NULL) receive the unsorted emission. */
void gso_bin(int64_t n, const int32_t *bounds, const float *depths, const int32_t *counts,
             int32_t tiles_w, int32_t num_tiles, int64_t *keys_out, int32_t *ids_out,
             int32_t *sorted_ids, int64_t *sorted_keys, int64_t *ranges) {
    int64_t total = gso_total(n, counts);
    uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(total ? total : 1));
    uint32_t *ids = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(total ? total : 1));
    int64_t offset = 0;
    for (int64_t g = 0; g < n; ++g) {
        int32_t count = counts[g];
        int32_t min_x = bounds[4 * g], max_x = bounds[4 * g + 1], min_y = bounds[4 * g + 2];
        int32_t width = max_x - min_x;
        uint32_t depth_bits = gso_f2u(depths[g]);
        for (int32_t local = 0; local < count; ++local) {
            int64_t tile = (int64_t)(min_y + local / width) * tiles_w + min_x + local % width;
            keys[offset + local] = ((uint64_t)tile << 32) | depth_bits;
            ids[offset + local] = (uint32_t)g;
        }
        offset += count;
    }
    if (keys_out) for (int64_t i = 0; i < total; ++i) keys_out[i] = (int64_t)keys[i];
    if (ids_out) for (int64_t i = 0; i < total; ++i) ids_out[i] = (int32_t)ids[i];
    /* Stable LSD radix sort on the 64-bit key, 16 bits per pass, skipping passes
     * whose digit is constant. Keys are non-negative, so unsigned order equals
     * the reference's signed int64 order. */
    uint64_t *k2 = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(total ? total : 1));
    uint32_t *v2 = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(total ? total : 1));
    int64_t *hist = (int64_t *)malloc(sizeof(int64_t) * 65536);
    for (int shift = 0; shift < 64; shift += 16) {
        memset(hist, 0, sizeof(int64_t) * 65536);
        for (int64_t i = 0; i < total; ++i) hist[(keys[i] >> shift) & 0xFFFF]++;
        int constant = 0;
        for (int d = 0; d < 65536; ++d) if (hist[d] == total) constant = 1;
        if (constant || total == 0) continue;
        int64_t run = 0;
        for (int d = 0; d < 65536; ++d) { int64_t c = hist[d]; hist[d] = run; run += c; }
        for (int64_t i = 0; i < total; ++i) {
            int64_t dst = hist[(keys[i] >> shift) & 0xFFFF]++;
            k2[dst] = keys[i];
            v2[dst] = ids[i];
        }
        uint64_t *tk = keys; keys = k2; k2 = tk;
        uint32_t *tv = ids; ids = v2; v2 = tv;
    }
    for (int64_t i = 0; i < total; ++i) sorted_ids[i] = (int32_t)ids[i];
    if (sorted_keys) for (int64_t i = 0; i < total; ++i) sorted_keys[i] = (int64_t)keys[i];
    int64_t *per_tile = (int64_t *)calloc((size_t)num_tiles + 1, sizeof(int64_t));
    for (int64_t i = 0; i < total; ++i) per_tile[keys[i] >> 32]++;
    int64_t end = 0;
    for (int32_t tile = 0; tile < num_tiles; ++tile) {
        ranges[2 * tile] = end;
        end += per_tile[tile];
        ranges[2 * tile + 1] = end;
    }
    free(per_tile); free(hist); free(k2); free(v2); free(keys); free(ids);
}

/* ---------------------------------------------------------------- composite */

static inline float pair_d2(float dx, float dy, float xx, float xy, float yy) {
    return fmaf(xx * dx, dx, fmaf((2.0f * xy) * dx, dy, (yy * dy) * dy));
}

/* A NaN distance (only reachable from a degenerate conic) contributes nothing. */
static inline float pair_probability(float d2, const gso_params *p) {
    if (d2 != d2) return 0.0f;
    return p->gaussian_mode ? gso_exp(-0.5f * d2) : (d2 <= p->cutoff ? 1.0f : 0.0f);
}

/* composite.py:25-107 for the tiles listed in `tiles` (all tiles when NULL). */
void gso_composite(const float *projected_mean, const float *inverse_covariance,
                   const float *projected_color, const float *projected_opacity,
                   const int32_t *gaussian_ids, const int64_t *ranges, const gso_params *p,
                   const int32_t *tiles, int32_t num_listed, float *image,
                   float *final_transmittance, int32_t *n_contributors) {
    const int ts = p->tile_size, tiles_w = p->width / ts, W = p->width;
    const int32_t num_tiles = tiles ? num_listed : (p->height / ts) * tiles_w;
    const float thr = p->opacity_threshold;
#pragma omp parallel for schedule(dynamic, 1)
    for (int32_t which = 0; which < num_tiles; ++which) {
        int32_t tile = tiles ? tiles[which] : which;
        int npix = ts * ts;
        float *T = (float *)malloc(sizeof(float) * npix * 4);
        float *C = T + npix;
        int32_t *contrib = (int32_t *)malloc(sizeof(int32_t) * npix);
        for (int q = 0; q < npix; ++q) { T[q] = 1.0f; C[3 * q] = C[3 * q + 1] = C[3 * q + 2] = 0.0f; contrib[q] = 0; }
        int x0 = (tile % tiles_w) * ts, y0 = (tile / tiles_w) * ts;
        for (int64_t k = ranges[2 * tile]; k < ranges[2 * tile + 1]; ++k) {
            int any_active = 0;
            for (int q = 0; q < npix; ++q) any_active |= (1.0f - T[q]) < thr;
            if (!any_active) break; /* composite.py:187-188 */
            int64_t g = gaussian_ids[k];
            float mx = projected_mean[3 * g], my = projected_mean[3 * g + 1];
            float xx = inverse_covariance[4 * g], xy = inverse_covariance[4 * g + 1],
                  yy = inverse_covariance[4 * g + 3];
            float o = projected_opacity[g];
            float cr = projected_color[3 * g], cg = projected_color[3 * g + 1],
                  cb = projected_color[3 * g + 2];
            for (int q = 0; q < npix; ++q) {
                float dx = (float)(x0 + q % ts) - mx;
                float dy = (float)(y0 + q / ts) - my;
                float prob = pair_probability(pair_d2(dx, dy, xx, xy, yy), p);
                float alpha = fminf(o * prob, 0.99f);
                alpha = alpha >= ALPHA_MIN ? alpha : 0.0f;
                int active = (1.0f - T[q]) < thr;
                contrib[q] += active;
                if (!active) continue;
                float weight = T[q] * alpha;
                C[3 * q] = fmaf(weight, cr, C[3 * q]);
                C[3 * q + 1] = fmaf(weight, cg, C[3 * q + 1]);
                C[3 * q + 2] = fmaf(weight, cb, C[3 * q + 2]);
                T[q] = T[q] * (1.0f - alpha);
            }
        }
        for (int q = 0; q < npix; ++q) {
            int64_t pix = (int64_t)(y0 + q / ts) * W + x0 + q % ts;
            image[3 * pix] = C[3 * q];
            image[3 * pix + 1] = C[3 * q + 1];
            image[3 * pix + 2] = C[3 * q + 2];
            final_transmittance[pix] = T[q];
            n_contributors[pix] = contrib[q];
        }
        free(T);
        free(contrib);
    }
}

/* ---------------------------------------------------------------- composite backward */

/* composite_bwd.py:47-277 (non-atomic variant): one 9-float row per
 * intersection [d mean_x, d mean_y, d conic_xx, d conic_xy (not doubled),
 * d conic_yy, d r, d g, d b, d opacity], summed over the tile's pixels in
 * pixel order, then accumulated into grad_projected [N, 9] in intersection
 * order like index_add_. The reverse scan is evaluated as a running suffix:
 * before entry k, (suffix_t, suffix_rgb) composite the entries behind k. */
void gso_composite_bwd(int64_t n, const float *projected_mean, const float *inverse_covariance,
                       const float *projected_color, const float *projected_opacity,
                       const int32_t *gaussian_ids, const int64_t *ranges, int64_t total,
                       const float *grad_image, const float *final_transmittance,
                       const int32_t *n_contributors, const gso_params *p,
                       const int32_t *tiles, int32_t num_listed, float *grad_projected) {
    /* `tiles` (optional) restricts the walk to the listed tiles; the caller
     * guarantees grad_image is zero elsewhere, where rows would be zero. */
    const int ts = p->tile_size, tiles_w = p->width / ts, W = p->width;
    const int32_t num_tiles = tiles ? num_listed : (p->height / ts) * tiles_w;
    const float thr = p->opacity_threshold;
    float *rows = (float *)calloc((size_t)(total ? total : 1) * 9, sizeof(float));
#pragma omp parallel for schedule(dynamic, 1)
    for (int32_t which = 0; which < num_tiles; ++which) {
        int32_t tile = tiles ? tiles[which] : which;
        int npix = ts * ts;
        float *st = (float *)malloc(sizeof(float) * npix * 4);
        float *sc = st + npix;
        int x0 = (tile % tiles_w) * ts, y0 = (tile / tiles_w) * ts;
        int32_t max_contrib = 0;
        for (int q = 0; q < npix; ++q) {
            int64_t pix = (int64_t)(y0 + q / ts) * W + x0 + q % ts;
            if (n_contributors[pix] > max_contrib) max_contrib = n_contributors[pix];
            st[q] = 1.0f;
            sc[3 * q] = sc[3 * q + 1] = sc[3 * q + 2] = 0.0f;
        }
        int64_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
        if (end > start + max_contrib) end = start + max_contrib; /* composite_bwd.py:81-83 */
        for (int64_t k = end - 1; k >= start; --k) {
            int64_t g = gaussian_ids[k];
            int64_t position = k - start;
            float mx = projected_mean[3 * g], my = projected_mean[3 * g + 1];
            float xx = inverse_covariance[4 * g], xy = inverse_covariance[4 * g + 1],
                  yy = inverse_covariance[4 * g + 3];
            float o = projected_opacity[g];
            float cr = projected_color[3 * g], cg = projected_color[3 * g + 1],
                  cb = projected_color[3 * g + 2];
            float *row = rows + 9 * k;
            for (int q = 0; q < npix; ++q) {
                int64_t pix = (int64_t)(y0 + q / ts) * W + x0 + q % ts;
                if (position >= n_contributors[pix]) continue;
                float dx = (float)(x0 + q % ts) - mx;
                float dy = (float)(y0 + q / ts) - my;
                float prob = pair_probability(pair_d2(dx, dy, xx, xy, yy), p);
                float alpha_raw = o * prob;
                float alpha = fminf(alpha_raw, 0.99f);
                if (!(alpha >= ALPHA_MIN)) continue; /* inactive: no gradient, suffix unchanged */
                float gr = grad_image[3 * pix], gg = grad_image[3 * pix + 1],
                      gb = grad_image[3 * pix + 2];
                float denominator = fmaxf(st[q] * (1.0f - alpha), 1e-4f);
                float forward = final_transmittance[pix] / denominator;
                int active = (1.0f - forward) < thr;
                float weight_grad = gr * (cr - sc[3 * q]);
                weight_grad += gg * (cg - sc[3 * q + 1]);
                weight_grad += gb * (cb - sc[3 * q + 2]);
                float grad_alpha = active ? forward * weight_grad : 0.0f;
                grad_alpha = alpha_raw < 0.99f ? grad_alpha : 0.0f;
                float probability_grad = grad_alpha * o;
                float grad_color = forward * alpha;
                /* ellipsoid mode: the indicator falloff has no gradient */
                float grad_distance = p->gaussian_mode ? -0.5f * prob * probability_grad : 0.0f;
                row[0] += -2.0f * grad_distance * (xx * dx + xy * dy);
                row[1] += -2.0f * grad_distance * (xy * dx + yy * dy);
                row[2] += grad_distance * dx * dx;
                row[3] += grad_distance * dx * dy;
                row[4] += grad_distance * dy * dy;
                row[5] += grad_color * gr;
                row[6] += grad_color * gg;
                row[7] += grad_color * gb;
                row[8] += grad_alpha * prob;
                float local_t = 1.0f - alpha;
                sc[3 * q] = fmaf(local_t, sc[3 * q], alpha * cr);
                sc[3 * q + 1] = fmaf(local_t, sc[3 * q + 1], alpha * cg);
                sc[3 * q + 2] = fmaf(local_t, sc[3 * q + 2], alpha * cb);
                st[q] = st[q] * local_t;
            }
        }
        free(st);
    }
    memset(grad_projected, 0, sizeof(float) * 9 * (size_t)n);
    for (int64_t k = 0; k < total; ++k) {
        int64_t g = gaussian_ids[k];
        for (int j = 0; j < 9; ++j) grad_projected[9 * g + j] += rows[9 * k + j];
    }
    free(rows);
}

/* ---------------------------------------------------------------- project backward */

static void project_bwd_one(int64_t i, const float *mean, const float *rotation,
                            const float *scale, const float *opacity, const float *color,
                            int32_t num_sh, const float *R, const float *t,
                            const float *inverse_covariance, const float *grad_projected,
                            const int32_t *counts, const gso_params *p, float *grad_mean,
                            float *grad_rotation, float *grad_scale, float *grad_opacity,
                            float *grad_color) {
    const int visible = counts[i] != 0;
    const float cr00 = R[0], cr01 = R[1], cr02 = R[2], cr10 = R[3], cr11 = R[4], cr12 = R[5],
                cr20 = R[6], cr21 = R[7], cr22 = R[8];
    const float tx = t[0], ty = t[1], tz = t[2];
    const float fx = p->fx, fy = p->fy, lim_x = p->bwd_lim_x, lim_y = p->bwd_lim_y;
    const float mx = mean[3 * i], my = mean[3 * i + 1], mz = mean[3 * i + 2];
    /* project_bwd.py:62-94 */
    float camera_x = mx * cr00 + my * cr01 + mz * cr02 + tx;
    float camera_y = mx * cr10 + my * cr11 + mz * cr12 + ty;
    float camera_z = mx * cr20 + my * cr21 + mz * cr22 + tz;
    float qw = rotation[4 * i], qx = rotation[4 * i + 1], qy = rotation[4 * i + 2],
          qz = rotation[4 * i + 3];
    float qnorm = sqrtf(qw * qw + qx * qx + qy * qy + qz * qz);
    float inverse_qnorm = 1.0f / qnorm;
    qw = qw * inverse_qnorm; qx = qx * inverse_qnorm; qy = qy * inverse_qnorm; qz = qz * inverse_qnorm;
    float r00 = 1.0f - 2.0f * (qy * qy + qz * qz), r01 = 2.0f * (qx * qy - qw * qz),
          r02 = 2.0f * (qx * qz + qw * qy);
    float r10 = 2.0f * (qx * qy + qw * qz), r11 = 1.0f - 2.0f * (qx * qx + qz * qz),
          r12 = 2.0f * (qy * qz - qw * qx);
    float r20 = 2.0f * (qx * qz - qw * qy), r21 = 2.0f * (qy * qz + qw * qx),
          r22 = 1.0f - 2.0f * (qx * qx + qy * qy);
    float depth = -camera_z;
    float inverse_z = 1.0f / depth;
    float normalized_x = camera_x * inverse_z, normalized_y = camera_y * inverse_z;
    float x_grad_mul = (normalized_x >= -lim_x && normalized_x <= lim_x) ? 1.0f : 0.0f;
    float y_grad_mul = (normalized_y >= -lim_y && normalized_y <= lim_y) ? 1.0f : 0.0f;
    float covariance_x = fminf(lim_x, fmaxf(-lim_x, normalized_x)) * depth;
    float covariance_y = fminf(lim_y, fmaxf(-lim_y, normalized_y)) * depth;
    float j00 = fx * inverse_z, j02 = fx * covariance_x * inverse_z * inverse_z;
    float j11 = -fy * inverse_z, j12 = -fy * covariance_y * inverse_z * inverse_z;
    /* project_bwd.py:96-114 */
    float jc00 = j00 * cr00 + j02 * cr20, jc01 = j00 * cr01 + j02 * cr21, jc02 = j00 * cr02 + j02 * cr22;
    float jc10 = j11 * cr10 + j12 * cr20, jc11 = j11 * cr11 + j12 * cr21, jc12 = j11 * cr12 + j12 * cr22;
    float sx = gso_exp(scale[3 * i]), sy = gso_exp(scale[3 * i + 1]), sz = gso_exp(scale[3 * i + 2]);
    float m0x = jc00 * r00 + jc01 * r10 + jc02 * r20, m0y = jc00 * r01 + jc01 * r11 + jc02 * r21,
          m0z = jc00 * r02 + jc01 * r12 + jc02 * r22;
    float m1x = jc10 * r00 + jc11 * r10 + jc12 * r20, m1y = jc10 * r01 + jc11 * r11 + jc12 * r21,
          m1z = jc10 * r02 + jc11 * r12 + jc12 * r22;
    float a00 = m0x * sx, a01 = m0y * sy, a02 = m0z * sz;
    float a10 = m1x * sx, a11 = m1y * sy, a12 = m1z * sz;
    /* project_bwd.py:116-152 */
    const float *gp = grad_projected + 9 * i;
    float inv00 = inverse_covariance[4 * i], inv01 = inverse_covariance[4 * i + 1];
    float inv10 = inv01, inv11 = inverse_covariance[4 * i + 3];
    float gi00 = gp[2], gi01 = gp[3], gi10 = gi01, gi11 = gp[4];
    float h00 = inv00 * gi00 + inv10 * gi10, h01 = inv00 * gi01 + inv10 * gi11;
    float h10 = inv01 * gi00 + inv11 * gi10, h11 = inv01 * gi01 + inv11 * gi11;
    float gcov00 = -(h00 * inv00 + h01 * inv10), gcov01 = -(h00 * inv01 + h01 * inv11);
    float gcov10 = -(h10 * inv00 + h11 * inv10), gcov11 = -(h10 * inv01 + h11 * inv11);
    float sym01 = gcov01 + gcov10;
    float ga00 = 2.0f * gcov00 * a00 + sym01 * a10, ga01 = 2.0f * gcov00 * a01 + sym01 * a11,
          ga02 = 2.0f * gcov00 * a02 + sym01 * a12;
    float ga10 = sym01 * a00 + 2.0f * gcov11 * a10, ga11 = sym01 * a01 + 2.0f * gcov11 * a11,
          ga12 = sym01 * a02 + 2.0f * gcov11 * a12;
    float gb00 = ga00 * sx, gb01 = ga01 * sy, gb02 = ga02 * sz;
    float gb10 = ga10 * sx, gb11 = ga11 * sy, gb12 = ga12 * sz;
    float grad_sx = ga00 * m0x + ga10 * m1x;
    float grad_sy = ga01 * m0y + ga11 * m1y;
    float grad_sz = ga02 * m0z + ga12 * m1z;
    /* project_bwd.py:154-189 */
    float gr00 = jc00 * gb00 + jc10 * gb10, gr01 = jc00 * gb01 + jc10 * gb11, gr02 = jc00 * gb02 + jc10 * gb12;
    float gr10 = jc01 * gb00 + jc11 * gb10, gr11 = jc01 * gb01 + jc11 * gb11, gr12 = jc01 * gb02 + jc11 * gb12;
    float gr20 = jc02 * gb00 + jc12 * gb10, gr21 = jc02 * gb01 + jc12 * gb11, gr22 = jc02 * gb02 + jc12 * gb12;
    float gqw = 2.0f * qz * (gr10 - gr01) + 2.0f * qy * (gr02 - gr20) + 2.0f * qx * (gr21 - gr12);
    float gqx = 2.0f * qy * (gr01 + gr10) + 2.0f * qz * (gr02 + gr20) + 2.0f * qw * (gr21 - gr12) -
                4.0f * qx * (gr11 + gr22);
    float gqy = 2.0f * qx * (gr01 + gr10) + 2.0f * qw * (gr02 - gr20) + 2.0f * qz * (gr12 + gr21) -
                4.0f * qy * (gr00 + gr22);
    float gqz = 2.0f * qw * (gr10 - gr01) + 2.0f * qx * (gr02 + gr20) + 2.0f * qy * (gr12 + gr21) -
                4.0f * qz * (gr00 + gr11);
    float dot_q = qw * gqw + qx * gqx + qy * gqy + qz * gqz;
    float gq_scale = 1.0f / qnorm;
    gqw = (gqw - qw * dot_q) * gq_scale;
    gqx = (gqx - qx * dot_q) * gq_scale;
    gqy = (gqy - qy * dot_q) * gq_scale;
    gqz = (gqz - qz * dot_q) * gq_scale;
    /* project_bwd.py:191-226 */
    float gpx = gp[0], gpy = gp[1];
    float gux = gpx * j00 + gpx * 0.0f;
    float guy = gpy * j11;
    float guz = -0.0f + gpx * j02 + gpy * j12;
    float mr0 = cr00 * r00 + cr01 * r10 + cr02 * r20, mr1 = cr00 * r01 + cr01 * r11 + cr02 * r21,
          mr2 = cr00 * r02 + cr01 * r12 + cr02 * r22;
    float nr0 = cr10 * r00 + cr11 * r10 + cr12 * r20, nr1 = cr10 * r01 + cr11 * r11 + cr12 * r21,
          nr2 = cr10 * r02 + cr11 * r12 + cr12 * r22;
    float kr0 = cr20 * r00 + cr21 * r10 + cr22 * r20, kr1 = cr20 * r01 + cr21 * r11 + cr22 * r21,
          kr2 = cr20 * r02 + cr21 * r12 + cr22 * r22;
    float gj_j00 = gb00 * mr0 + gb01 * mr1 + gb02 * mr2;
    float gj_j02 = gb00 * kr0 + gb01 * kr1 + gb02 * kr2;
    float gj_j11 = gb10 * nr0 + gb11 * nr1 + gb12 * nr2;
    float gj_j12 = gb10 * kr0 + gb11 * kr1 + gb12 * kr2;
    gux += x_grad_mul * gj_j02 * (fx * inverse_z * inverse_z);
    guy += y_grad_mul * gj_j12 * (-fy * inverse_z * inverse_z);
    float inverse_z3 = inverse_z * inverse_z * inverse_z;
    guz += gj_j00 * (fx * inverse_z * inverse_z) + gj_j02 * 2.0f * fx * covariance_x * inverse_z3;
    guz += gj_j11 * (-fy * inverse_z * inverse_z) - gj_j12 * 2.0f * fy * covariance_y * inverse_z3;
    float gmx = gux * cr00 + guy * cr10 + guz * cr20;
    float gmy = gux * cr01 + guy * cr11 + guz * cr21;
    float gmz = gux * cr02 + guy * cr12 + guz * cr22;
    /* project_bwd.py:228-318 (degree <= 3); degree 4 (coefficients 16..24)
     * differentiates the forward basis (project.py:51-61) the same way,
     * where the reference's backward stops at 16 (project_bwd.py:33). */
    float dx = mx + cr00 * tx + cr10 * ty + cr20 * tz;
    float dy = my + cr01 * tx + cr11 * ty + cr21 * tz;
    float dz = mz + cr02 * tx + cr12 * ty + cr22 * tz;
    float norm = sqrtf(dx * dx + dy * dy + dz * dz);
    float x = dx / norm, y = dy / norm, z = dz / norm;
    float xx = x * x, yy = y * y, zz = z * z;
    float basis[25], dbx[25], dby[25], dbz[25];
    memset(dbx, 0, sizeof dbx); memset(dby, 0, sizeof dby); memset(dbz, 0, sizeof dbz);
    basis[0] = 0.28209479177387814f;
    basis[1] = -0.4886025119029199f * y;
    basis[2] = 0.4886025119029199f * z;
    basis[3] = -0.4886025119029199f * x;
    basis[4] = 1.0925484305920792f * x * y;
    basis[5] = -1.0925484305920792f * y * z;
    basis[6] = 0.31539156525252005f * (2.0f * zz - xx - yy);
    basis[7] = -1.0925484305920792f * x * z;
    basis[8] = 0.5462742152960396f * (xx - yy);
    basis[9] = -0.5900435899266435f * y * (3.0f * xx - yy);
    basis[10] = 2.890611442640554f * x * y * z;
    basis[11] = -0.4570457994644655f * y * (4.0f * zz - xx - yy);
    basis[12] = 0.3731763325901154f * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    basis[13] = -0.4570457994644655f * x * (4.0f * zz - xx - yy);
    basis[14] = 1.445305721320277f * z * (xx - yy);
    basis[15] = -0.5900435899266435f * x * (xx - 3.0f * yy);
    dbx[3] = -0.4886025119029199f;
    dby[1] = -0.4886025119029199f;
    dbz[2] = 0.4886025119029199f;
    dbx[4] = 1.0925484305920792f * y;
    dby[4] = 1.0925484305920792f * x;
    dby[5] = -1.0925484305920792f * z;
    dbz[5] = -1.0925484305920792f * y;
    dbx[6] = -0.6307831301050401f * x;
    dby[6] = -0.6307831301050401f * y;
    dbz[6] = 1.2615662610100802f * z;
    dbx[7] = -1.0925484305920792f * z;
    dbz[7] = -1.0925484305920792f * x;
    dbx[8] = 1.0925484305920792f * x;
    dby[8] = -1.0925484305920792f * y;
    dbx[9] = -3.540261539559861f * x * y;
    dby[9] = -1.7701307697799305f * (xx - yy);
    dbx[10] = 2.890611442640554f * y * z;
    dby[10] = 2.890611442640554f * x * z;
    dbz[10] = 2.890611442640554f * x * y;
    dbx[11] = 0.914091599852931f * x * y;
    dby[11] = -0.4570457994644655f * (4.0f * zz - xx - 3.0f * yy);
    dbz[11] = -3.656366399411724f * y * z;
    dbx[12] = -2.2390579955366924f * x * z;
    dby[12] = -2.2390579955366924f * y * z;
    dbz[12] = 0.3731763325901154f * (6.0f * zz - 3.0f * xx - 3.0f * yy);
    dbx[13] = -0.4570457994644655f * (4.0f * zz - 3.0f * xx - yy);
    dby[13] = 0.914091599852931f * x * y;
    dbz[13] = -3.656366399411724f * x * z;
    dbx[14] = 2.890611442640554f * x * z;
    dby[14] = -2.890611442640554f * y * z;
    dbz[14] = 1.445305721320277f * (xx - yy);
    dbx[15] = -1.7701307697799305f * (xx - yy);
    dby[15] = 3.540261539559861f * x * y;
    if (num_sh > 16) {
        basis[16] = 2.5033429417967046f * x * y * (xx - yy);
        basis[17] = -1.7701307697799304f * y * z * (3.0f * xx - yy);
        basis[18] = 0.9461746957575601f * x * y * (7.0f * zz - 1.0f);
        basis[19] = -0.6690465435572892f * y * z * (7.0f * zz - 3.0f);
        basis[20] = 0.10578554691520431f * (zz * (35.0f * zz - 30.0f) + 3.0f);
        basis[21] = -0.6690465435572892f * x * z * (7.0f * zz - 3.0f);
        basis[22] = 0.47308734787878004f * (xx - yy) * (7.0f * zz - 1.0f);
        basis[23] = -1.7701307697799304f * x * z * (xx - 3.0f * yy);
        basis[24] = 0.6258357354491761f * (xx * (xx - 3.0f * yy) - yy * (3.0f * xx - yy));
        dbx[16] = 2.5033429417967046f * y * (3.0f * xx - yy);
        dby[16] = 2.5033429417967046f * x * (xx - 3.0f * yy);
        dbx[17] = -10.620784618679583f * x * y * z;
        dby[17] = -5.310392309339791f * z * (xx - yy);
        dbz[17] = -1.7701307697799304f * y * (3.0f * xx - yy);
        dbx[18] = 0.9461746957575601f * y * (7.0f * zz - 1.0f);
        dby[18] = 0.9461746957575601f * x * (7.0f * zz - 1.0f);
        dbz[18] = 13.246445740605841f * x * y * z;
        dby[19] = -0.6690465435572892f * z * (7.0f * zz - 3.0f);
        dbz[19] = -0.6690465435572892f * y * (21.0f * zz - 3.0f);
        dbz[20] = 0.10578554691520431f * z * (140.0f * zz - 60.0f);
        dbx[21] = -0.6690465435572892f * z * (7.0f * zz - 3.0f);
        dbz[21] = -0.6690465435572892f * x * (21.0f * zz - 3.0f);
        dbx[22] = 0.9461746957575601f * x * (7.0f * zz - 1.0f);
        dby[22] = -0.9461746957575601f * y * (7.0f * zz - 1.0f);
        dbz[22] = 6.623222870302921f * z * (xx - yy);
        dbx[23] = -5.310392309339791f * z * (xx - yy);
        dby[23] = 10.620784618679583f * x * y * z;
        dbz[23] = -1.7701307697799304f * x * (xx - 3.0f * yy);
        dbx[24] = 2.5033429417967046f * x * (xx - 3.0f * yy);
        dby[24] = 2.5033429417967046f * y * (yy - 3.0f * xx);
    }
    const int kmax = num_sh;
    const float *coefficients = color + i * (int64_t)num_sh * 3;
    float *gcol = grad_color + i * (int64_t)num_sh * 3;
    float gdx = 0.0f, gdy = 0.0f, gdz = 0.0f;
    for (int c = 0; c < 3; ++c) {
        float raw = 0.0f, sdx = 0.0f, sdy = 0.0f, sdz = 0.0f;
        for (int k = 0; k < kmax; ++k) {
            float coef = coefficients[3 * k + c];
            raw = fmaf(coef, basis[k], raw);
            sdx = fmaf(coef, dbx[k], sdx);
            sdy = fmaf(coef, dby[k], sdy);
            sdz = fmaf(coef, dbz[k], sdz);
        }
        raw = raw + 0.5f;
        float gc = gp[5 + c] * (raw > 0.0f ? 1.0f : 0.0f);
        for (int k = 0; k < kmax; ++k) gcol[3 * k + c] = visible ? gc * basis[k] : 0.0f;
        gdx += gc * sdx;
        gdy += gc * sdy;
        gdz += gc * sdz;
    }
    float dot_d = x * gdx + y * gdy + z * gdz;
    gdx = (gdx - x * dot_d) / norm;
    gdy = (gdy - y * dot_d) / norm;
    gdz = (gdz - z * dot_d) / norm;
    gmx += gdx; gmy += gdy; gmz += gdz;
    /* project_bwd.py:320-334 */
    float po = gso_sigmoid(opacity[i]);
    float go = gp[8] * po * (1.0f - po);
    grad_mean[3 * i] = visible ? gmx : 0.0f;
    grad_mean[3 * i + 1] = visible ? gmy : 0.0f;
    grad_mean[3 * i + 2] = visible ? gmz : 0.0f;
    grad_rotation[4 * i] = visible ? gqw : 0.0f;
    grad_rotation[4 * i + 1] = visible ? gqx : 0.0f;
    grad_rotation[4 * i + 2] = visible ? gqy : 0.0f;
    grad_rotation[4 * i + 3] = visible ? gqz : 0.0f;
    grad_scale[3 * i] = visible ? grad_sx * sx : 0.0f;
    grad_scale[3 * i + 1] = visible ? grad_sy * sy : 0.0f;
    grad_scale[3 * i + 2] = visible ? grad_sz * sz : 0.0f;
    grad_opacity[i] = visible ? go : 0.0f;
}

void gso_project_bwd(int64_t n, const float *mean, const float *rotation, const float *scale,
                     const float *opacity, const float *color, int32_t num_sh, const float *R,
                     const float *t, const float *inverse_covariance,
                     const float *grad_projected, const int32_t *counts, const gso_params *p,
                     float *grad_mean, float *grad_rotation, float *grad_scale,
                     float *grad_opacity, float *grad_color) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        project_bwd_one(i, mean, rotation, scale, opacity, color, num_sh, R, t,
                        inverse_covariance, grad_projected, counts, p, grad_mean, grad_rotation,
                        grad_scale, grad_opacity, grad_color);
}

/* Deterministic exp/log exposed for the bitwise CPU/GPU agreement test. */
/* ---------------------------------------------------------------- optimizer step */

/* torch.optim.Adam's foreach step (eps 1e-15 and one group per parameter as
 * training/train.py:111-118 builds them) followed by noise_splats
 * (training/utils.py:50-62) on the updated parameters. Scalars arrive folded
 * as torch folds them (double, then float). Per element, in torch's order:
 *   m = m + w1 (g - m); v = v b2; v = v + w2 (g g);
 *   p = p + neg_step (m / (sqrt(v) / bias2_sqrt + eps)). */
typedef struct gso_adam_params {
    float lerp_weight, beta2, sq_weight, eps;
    float neg_step_size[5];
    float bias2_sqrt[5];
    float noise_lr, position_lr;
} gso_adam_params;

static float adam_one(float p, float g, float *m, float *v, float neg_step, float bias2_sqrt,
                      const gso_adam_params *h) {
    *m = *m + h->lerp_weight * (g - *m);
    *v = *v * h->beta2;
    *v = *v + h->sq_weight * (g * g);
    float d = sqrtf(*v) / bias2_sqrt + h->eps;
    return p + neg_step * (*m / d);
}

static float sigmoidf_det(float x) { return 1.0f / (1.0f + gso_exp(-x)); }

/* params/grads/m/v: pointers to mean, rotation, scale, opacity, color (a NULL
 * gradient skips that parameter); randn [N,3] or NULL for no noise. */
void gso_adam_step(int64_t n, int32_t num_sh, float *const *params, const float *const *grads,
                   float *const *m, float *const *v, const gso_adam_params *h,
                   const float *randn) {
    static const int widths[4] = {3, 4, 3, 1};
    for (int k = 0; k < 4; ++k) {
        if (!grads[k]) continue;
        for (int64_t e = 0; e < n * widths[k]; ++e)
            params[k][e] = adam_one(params[k][e], grads[k][e], &m[k][e], &v[k][e],
                                    h->neg_step_size[k], h->bias2_sqrt[k], h);
    }
    if (grads[4]) {
        for (int64_t e = 0; e < n * 3 * (int64_t)num_sh; ++e)
            params[4][e] = adam_one(params[4][e], grads[4][e], &m[4][e], &v[4][e],
                                    h->neg_step_size[4], h->bias2_sqrt[4], h);
    }
    if (!randn) return;
    for (int64_t i = 0; i < n; ++i) {
        const float *r4 = params[1] + 4 * i, *sc = params[2] + 3 * i;
        float norm = sqrtf(((r4[0] * r4[0] + r4[1] * r4[1]) + r4[2] * r4[2]) + r4[3] * r4[3]);
        float inv = fmaxf(norm, 1e-12f);
        float w = r4[0] / inv, x = r4[1] / inv, y = r4[2] / inv, z = r4[3] / inv;
        float r[3][3] = {
            {1.0f - 2.0f * (y * y + z * z), 2.0f * (x * y - w * z), 2.0f * (x * z + w * y)},
            {2.0f * (x * y + w * z), 1.0f - 2.0f * (x * x + z * z), 2.0f * (y * z - w * x)},
            {2.0f * (x * z - w * y), 2.0f * (y * z + w * x), 1.0f - 2.0f * (x * x + y * y)}};
        float s[3] = {gso_exp(sc[0]), gso_exp(sc[1]), gso_exp(sc[2])};
        float f[3][3];
        for (int a = 0; a < 3; ++a)
            for (int b = 0; b < 3; ++b) f[a][b] = r[a][b] * s[b];
        float gate = sigmoidf_det(100.0f * (1.0f - sigmoidf_det(params[3][i]) - 0.995f));
        float nz[3];
        for (int k = 0; k < 3; ++k) nz[k] = ((randn[3 * i + k] * gate) * h->noise_lr) * h->position_lr;
        for (int a = 0; a < 3; ++a) {
            float shift = 0.0f;
            for (int b = 0; b < 3; ++b) {
                float cov = (f[a][0] * f[b][0] + f[a][1] * f[b][1]) + f[a][2] * f[b][2];
                shift = b == 0 ? cov * nz[0] : shift + cov * nz[b];
            }
            params[0][3 * i + a] = params[0][3 * i + a] + shift;
        }
    }
}

/* Relocation (training/utils.py:120-145 with :94-101 and the moment reset of
 * :187-193). Parents in index order take consecutive output slots
 * (parents.repeat_interleave(copies)); slot j writes row output_indices[j], or
 * output_base + j when output_indices is NULL. normalize_copies with copies =
 * count + 1 clamped to 51: o' = 1 - (1 - o)^(1/copies), sum = sum over d of
 * C(copies, d) (-1)^(d-1) o'^d / sqrt(d), scale' = scale o / sum, opacity' =
 * clamp(o', 0.005, 1 - 1e-6) -- evaluated in double, each output rounded to
 * float once (the reference chains float32 operations; its results differ
 * from these by its rounding). moments[10] = exp_avg then exp_avg_sq of mean,
 * rotation, scale, opacity, colour (NULL entries skipped). Returns error bits:
 * 1 negative count, 2 counts not adding up to num_outputs, 4 output row out
 * of range (those slots are skipped). */
static void zero_moment_row(float *const *moments, int64_t row, int32_t num_sh) {
  static const int widths[5] = {3, 4, 3, 1, 0};
  for (int set = 0; set < 2; ++set)
    for (int k = 0; k < 5; ++k) {
      float *m = moments[5 * set + k];
      if (!m) continue;
      const int w = k == 4 ? 3 * num_sh : widths[k];
      for (int e = 0; e < w; ++e) m[row * w + e] = 0.0f;
    }
}

int gso_relocate(int64_t n_src, int64_t n_rows, int32_t num_sh, const int64_t *counts,
                 int64_t num_outputs, const int64_t *output_indices, int64_t output_base,
                 float *mean, float *rotation, float *scale, float *opacity, float *color,
                 float *normals, float *const *moments) {
  int error = 0;
  int64_t total = 0;
  for (int64_t i = 0; i < n_src; ++i) {
    if (counts[i] < 0) error |= 1;
    total += counts[i] > 0 ? counts[i] : 0;
  }
  if (total != num_outputs) error |= 2;
  const int w = 3 * num_sh;
  int64_t slot = 0;
  for (int64_t parent = 0; parent < n_src; ++parent) {
    const int64_t count = counts[parent] > 0 ? counts[parent] : 0;
    if (count == 0) continue;
    const int copies = count + 1 < 51 ? (int)(count + 1) : 51;
    const double o = 1.0 / (1.0 + exp(-(double)opacity[parent]));
    const double new_opacity = 1.0 - pow(1.0 - o, 1.0 / copies);
    double sum = 0.0, binomial = 1.0, power = 1.0;
    for (int d = 1; d <= copies; ++d) {
      binomial = binomial * (copies - d + 1) / d;
      power = power * new_opacity;
      const double term = binomial * power / sqrt((double)d);
      sum = (d & 1) ? sum + term : sum - term;
    }
    const double ratio = o / sum;
    const double p = fmin(fmax(new_opacity, (double)0.005f), (double)(float)(1.0 - 1e-6));
    const float logit = (float)log(p / (1.0 - p));
    float log_scale[3];
    for (int a = 0; a < 3; ++a) log_scale[a] = (float)log(exp((double)scale[3 * parent + a]) * ratio);
    for (int64_t j = slot; j < slot + count; ++j) {
      if (j >= num_outputs) {
        error |= 2;
        break;
      }
      const int64_t row = output_indices ? output_indices[j] : output_base + j;
      if (row < 0 || row >= n_rows) {
        error |= 4;
        continue;
      }
      memcpy(mean + 3 * row, mean + 3 * parent, 3 * sizeof(float));
      memcpy(rotation + 4 * row, rotation + 4 * parent, 4 * sizeof(float));
      memcpy(color + row * w, color + parent * w, (size_t)w * sizeof(float));
      if (normals) memcpy(normals + 3 * row, normals + 3 * parent, 3 * sizeof(float));
      opacity[row] = logit;
      for (int a = 0; a < 3; ++a) scale[3 * row + a] = log_scale[a];
      zero_moment_row(moments, row, num_sh);
    }
    slot += count;
    opacity[parent] = logit;
    for (int a = 0; a < 3; ++a) scale[3 * parent + a] = log_scale[a];
    zero_moment_row(moments, parent, num_sh);
  }
  return error;
}

void gso_exp_array(int64_t n, const float *x, float *y) { for (int64_t i = 0; i < n; ++i) y[i] = gso_exp(x[i]); }
void gso_log_array(int64_t n, const float *x, float *y) { for (int64_t i = 0; i < n; ++i) y[i] = gso_log(x[i]); }
