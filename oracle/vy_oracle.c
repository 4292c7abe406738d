/*
 * vy_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C restatement, on the CPU, of the arithmetic archish9/Vaayu holds its fused
 * packed-int4 MoE expert kernels to.  Only the test suite, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / `--impl reference` leg load this library, and only as the
 * checker or the timed CPU baseline: the CUDA product path never calls it.
 *
 * What each function restates (paths are inside the reference project):
 *
 *   vyo_dequant_flat   vaayu/moe_patch.py:750-769 `_fused_dequant_kernel` (and the blob walk
 *                      of `dequantize_expert_blob`, :849-864): code = (word >> b*j) & mask,
 *                      w = act(act(code - 2^(b-1)) * act(scale[i / gs])).
 *   vyo_dequant_role   vaayu/moe_patch.py:713-744 `dequantize_packed_weight` (symmetric) plus the
 *                      asymmetric extension w = act(act(u - z) * act(s)), z unpacked from
 *                      compressed-tensors' row-packed zero points (pack_to_int32 packed_dim=0).
 *   vyo_moe_layer      vaayu/packed_expert_kernels.py:785-814 `stock_experts_prefill` with
 *                      `linear=_linear_fp32` (:780-782), which for one token equals
 *                      `stock_experts_decode` (:399-410): per live expert in ascending id,
 *                      g = act(x.Wg), u = act(x.Wu), a = act(silu(g)), h = act(a*u),
 *                      y = act(h.Wd), c = fp32(y) * w (act-rounded when w is the act dtype),
 *                      out[t] = sum of c over the token's slots in ascending expert id
 *                      (accumulate_expert_outputs, vaayu/moe_patch.py:914-940).  Dot products
 *                      are summed in double and rounded once (double -> float -> act), the
 *                      "correctly rounded" replay tests/test_packed_prefill_kernels.py:117-134
 *                      holds the reference kernels to.
 *   vyo_fp8_dequant    vaayu/model_code/deepseek_v4/modeling_deepseek_v4.py:228-240
 *                      `dequantize_block_scaled`: bf16(float(w) * float(scale[tile])).
 *   vyo_fp4_dequant    no reference function (parity unpinned): e2m1 magnitudes
 *                      {0,.5,1,1.5,2,3,4,6} (OCP MX spec), sign bit 3, low nibble first, times
 *                      an e4m3 scale per `gs` elements of a row, rounded to bf16.
 *   vyo_fp_gemv        no reference function: out[t,n] = bf16(sum_k deq(W)[n,k] * x[t,k]),
 *                      the dequantised weight as `vyo_fp8_dequant`/`vyo_fp4_dequant` give it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { VYO_BF16 = 0, VYO_F16 = 1, VYO_F32 = 2, VYO_E4M3 = 3, VYO_E8M0 = 4 };

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* fp32 -> bf16 bits, round to nearest even; a NaN stays a (quiet) NaN. */
uint16_t vyo_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if (f != f) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

float vyo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        float v = (float)m * 5.9604644775390625e-08f;   /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13) | (m ? 0x400000u : 0u));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* fp32 -> fp16 bits, IEEE round to nearest even, overflow to inf, NaN kept. */
uint16_t vyo_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u)
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? (0x200u | ((ax >> 13) & 0x3FFu)) : 0u));
    int32_t e = (int32_t)(ax >> 23) - 127 + 15;
    uint32_t mant = ax & 0x7FFFFFu;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {                                   /* half subnormal or zero */
        if (e < -10) return (uint16_t)sign;         /* below half of the smallest subnormal */
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);        /* 14..24 */
        uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;   /* carry may reach inf: correct */
    return (uint16_t)(sign | h);
}

static inline float f16_to_f32(uint16_t h) { return vyo_f16_to_f32(h); }

/* `v` rounded to the dtype `code` names, held in a float. */
static inline float round_act(float v, int code) {
    if (code == VYO_BF16) return bf16_to_f32(vyo_f32_to_bf16(v));
    if (code == VYO_F16) return f16_to_f32(vyo_f32_to_f16(v));
    return v;
}

float vyo_e4m3_to_f32(uint8_t b) {
    uint32_t s = b >> 7, e = (b >> 3) & 0xFu, m = b & 7u;
    float v;
    if (e == 15 && m == 7) return u2f(0x7FC00000u | (s << 31));
    if (e == 0) v = (float)m * 0.001953125f;          /* m/8 * 2^-6 */
    else v = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
    return s ? -v : v;
}

static inline float e8m0_to_f32(uint8_t b) {
    if (b == 255) return u2f(0x7FC00000u);
    return ldexpf(1.0f, (int)b - 127);
}

static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
static inline float e2m1_to_f32(uint32_t nib) {
    float v = kE2M1[nib & 7u];
    return (nib & 8u) ? -v : v;
}

static inline float load_val(const void* p, int code, int64_t i) {
    switch (code) {
    case VYO_BF16: return bf16_to_f32(((const uint16_t*)p)[i]);
    case VYO_F16: return f16_to_f32(((const uint16_t*)p)[i]);
    case VYO_F32: return ((const float*)p)[i];
    case VYO_E4M3: return vyo_e4m3_to_f32(((const uint8_t*)p)[i]);
    case VYO_E8M0: return e8m0_to_f32(((const uint8_t*)p)[i]);
    default: return NAN;
    }
}

static inline void store_val(void* p, int code, int64_t i, float v) {
    if (code == VYO_BF16) ((uint16_t*)p)[i] = vyo_f32_to_bf16(v);
    else if (code == VYO_F16) ((uint16_t*)p)[i] = vyo_f32_to_f16(v);
    else ((float*)p)[i] = v;
}

/* -------------------------------------------------------------------------------------- */
/* int4 / int-b dequant                                                                    */
/* -------------------------------------------------------------------------------------- */

/* Flat blob stream: element i = code i of the stream, scaled by scale[i / gs]. */
int vyo_dequant_flat(const int32_t* packed, int64_t n_words, int bits, const void* scale,
                     int scale_code, int gs, int act_code, void* out) {
    if (bits <= 0 || bits > 8 || 32 % bits || gs <= 0) return -1;
    const int per = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const float off = (float)(1 << (bits - 1));
    for (int64_t w = 0; w < n_words; ++w) {
        uint32_t word = (uint32_t)packed[w];
        for (int j = 0; j < per; ++j) {
            int64_t i = w * per + j;
            float code = round_act((float)((word >> (bits * j)) & mask) - off, act_code);
            float s = round_act(load_val(scale, scale_code, i / gs), act_code);
            store_val(out, act_code, i, round_act(code * s, act_code));
        }
    }
    return 0;
}

/* Code of element (r, c) of a [rows, cols] role packed along columns. */
static inline uint32_t code_at(const int32_t* packed, int64_t words_per_row, int bits,
                               int64_t r, int64_t c) {
    const int per = 32 / bits;
    uint32_t word = (uint32_t)packed[r * words_per_row + c / per];
    return (word >> (bits * (c % per))) & ((1u << bits) - 1u);
}

/* Stored zero code of (row r, group g): compressed-tensors packs zero points along rows. */
static inline uint32_t zero_at(const int32_t* zero, int64_t groups, int bits, int64_t r, int64_t g) {
    const int per = 32 / bits;
    uint32_t word = (uint32_t)zero[(r / per) * groups + g];
    return (word >> (bits * (r % per))) & ((1u << bits) - 1u);
}

/* Row `r` of one role dequantised into `dst` (floats holding act-rounded values). */
static void dequant_row(const int32_t* packed, const void* scale, int scale_code,
                        const int32_t* zero, int64_t rows, int64_t cols, int bits, int gs,
                        int act_code, int64_t r, float* dst) {
    (void)rows;
    const int64_t wpr = cols * bits / 32, groups = cols / gs;
    const float off = (float)(1 << (bits - 1));
    for (int64_t c = 0; c < cols; ++c) {
        int64_t g = c / gs;
        float u = (float)code_at(packed, wpr, bits, r, c);
        float z = zero ? (float)zero_at(zero, groups, bits, r, g) : off;
        float s = round_act(load_val(scale, scale_code, r * groups + g), act_code);
        dst[c] = round_act(round_act(u - z, act_code) * s, act_code);
    }
}

int vyo_dequant_role(const int32_t* packed, int64_t rows, int64_t cols, int bits,
                     const void* scale, int scale_code, int gs, const int32_t* zero,
                     int act_code, void* out) {
    if (bits <= 0 || bits > 8 || 32 % bits || gs <= 0 || cols % gs || (cols * bits) % 32)
        return -1;
    float* row = (float*)malloc(sizeof(float) * (size_t)cols);
    if (!row) return -2;
    for (int64_t r = 0; r < rows; ++r) {
        dequant_row(packed, scale, scale_code, zero, rows, cols, bits, gs, act_code, r, row);
        for (int64_t c = 0; c < cols; ++c) store_val(out, act_code, r * cols + c, row[c]);
    }
    free(row);
    return 0;
}

/* -------------------------------------------------------------------------------------- */
/* The MoE expert layer                                                                    */
/* -------------------------------------------------------------------------------------- */

typedef struct {
    int32_t hidden, inter, bits, group_size;
    int32_t scale_code, act_code, w_code, has_zero;
    /* role order 0 gate [I,H], 1 up [I,H], 2 down [H,I]: offsets into one expert's streams */
    int64_t w_off[3];   /* int32 words   */
    int64_t s_off[3];   /* scale elements */
    int64_t z_off[3];   /* int32 words of the row-packed zero points */
} vyo_geom;

static inline const void* scale_at(const void* base, int code, int64_t off) {
    size_t es = code == VYO_F32 ? 4 : 2;
    return (const char*)base + (size_t)off * es;
}

/*
 * out[T, hidden] (fp32) = the routed-expert sum of one MoE layer.
 *   x        [T, hidden] act dtype, row stride x_stride elements
 *   eidx     [T*K] expert index of each (token, slot) row (row = t*K + k), 0 <= e < n_experts
 *   rw       routing weights in w_code; row j uses rw[w_index ? w_index[j] : j]
 *   table    [n_experts][3] addresses: packed int32 stream, scale stream, zero stream (or 0)
 *   h_out    optional [T*K, inter] act dtype: each row's SiLU(gate)*up
 *   y_out    optional [T*K, hidden] fp32: each row's weighted contribution
 *   h_in     optional [T*K, inter] act dtype: use this h instead of computing it
 */
int vyo_moe_layer(const vyo_geom* g, const void* x, int64_t x_stride, int32_t T,
                  const int64_t* eidx, int32_t K, const void* rw, const int32_t* w_index,
                  const int64_t* table, int32_t n_experts, float* out, int64_t out_stride,
                  void* h_out, float* y_out, const void* h_in, int32_t n_threads) {
    const int64_t H = g->hidden, I = g->inter, n = (int64_t)T * K;
    const int act = g->act_code, bits = g->bits, gs = g->group_size;
    if (T < 0 || K <= 0 || H <= 0 || I <= 0 || bits <= 0 || 32 % bits || gs <= 0) return -1;
    if (H % gs || I % gs) return -1;
    for (int64_t j = 0; j < n; ++j)
        if (eidx[j] < 0 || eidx[j] >= n_experts) return -3;
    if (n == 0) return 0;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
    /* Stable grouping of rows by expert (ascending id, then row). */
    int64_t* count = (int64_t*)calloc((size_t)n_experts + 1, sizeof(int64_t));
    int64_t* order = (int64_t*)malloc(sizeof(int64_t) * (size_t)n);
    float* xf = (float*)malloc(sizeof(float) * (size_t)(T * H));
    float* hbuf = (float*)malloc(sizeof(float) * (size_t)(n * I));
    float* ybuf = (float*)malloc(sizeof(float) * (size_t)(n * H));
    int64_t* live = (int64_t*)malloc(sizeof(int64_t) * (size_t)n_experts);
    if (!count || !order || !xf || !hbuf || !ybuf || !live) {
        free(count); free(order); free(xf); free(hbuf); free(ybuf); free(live);
        return -2;
    }
    for (int64_t j = 0; j < n; ++j) count[eidx[j] + 1]++;
    for (int64_t e = 0; e < n_experts; ++e) count[e + 1] += count[e];
    {
        int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)n_experts);
        memcpy(fill, count, sizeof(int64_t) * (size_t)n_experts);
        for (int64_t j = 0; j < n; ++j) order[fill[eidx[j]]++] = j;
        free(fill);
    }
    int64_t n_live = 0;
    for (int64_t e = 0; e < n_experts; ++e)
        if (count[e + 1] > count[e]) live[n_live++] = e;
    for (int64_t t = 0; t < T; ++t)
        for (int64_t k = 0; k < H; ++k)
            xf[t * H + k] = load_val((const char*)x, act, t * x_stride + k);

    /* Phase 1: h = act(act(silu(act(x.Wg))) * act(x.Wu)) for every routed row -- or, to check
     * the down stage alone, the caller's h (h_in, act dtype [T*K, I]). */
    if (h_in)
        for (int64_t j = 0; j < n * I; ++j) hbuf[j] = load_val(h_in, act, j);
#pragma omp parallel if (!h_in)
    if (!h_in) {
        float* wg = (float*)malloc(sizeof(float) * (size_t)H);
        float* wu = (float*)malloc(sizeof(float) * (size_t)H);
#pragma omp for schedule(dynamic, 4)
        for (int64_t it = 0; it < n_live * I; ++it) {
            int64_t e = live[it / I], r = it % I;
            const int32_t* pk = (const int32_t*)(intptr_t)table[e * 3 + 0];
            const void* sc = (const void*)(intptr_t)table[e * 3 + 1];
            const int32_t* zp = g->has_zero ? (const int32_t*)(intptr_t)table[e * 3 + 2] : NULL;
            dequant_row(pk + g->w_off[0], scale_at(sc, g->scale_code, g->s_off[0]), g->scale_code,
                        zp ? zp + g->z_off[0] : NULL, I, H, bits, gs, act, r, wg);
            dequant_row(pk + g->w_off[1], scale_at(sc, g->scale_code, g->s_off[1]), g->scale_code,
                        zp ? zp + g->z_off[1] : NULL, I, H, bits, gs, act, r, wu);
            for (int64_t q = count[e]; q < count[e + 1]; ++q) {
                int64_t j = order[q];
                const float* xt = xf + (j / K) * H;
                double ag = 0.0, au = 0.0;
                for (int64_t k = 0; k < H; ++k) {
                    ag += (double)wg[k] * (double)xt[k];
                    au += (double)wu[k] * (double)xt[k];
                }
                float gv = round_act((float)ag, act), uv = round_act((float)au, act);
                float av = round_act(gv / (1.0f + expf(-gv)), act);
                hbuf[j * I + r] = round_act(av * uv, act);
            }
        }
        free(wg);
        free(wu);
    }
    /* Phase 2: y = act(h.Wd); c = y * w (rounded to act when w is the act dtype). */
    const int w_round = (g->w_code == act) && act != VYO_F32;
#pragma omp parallel
    {
        float* wd = (float*)malloc(sizeof(float) * (size_t)I);
#pragma omp for schedule(dynamic, 8)
        for (int64_t it = 0; it < n_live * H; ++it) {
            int64_t e = live[it / H], r = it % H;
            const int32_t* pk = (const int32_t*)(intptr_t)table[e * 3 + 0];
            const void* sc = (const void*)(intptr_t)table[e * 3 + 1];
            const int32_t* zp = g->has_zero ? (const int32_t*)(intptr_t)table[e * 3 + 2] : NULL;
            dequant_row(pk + g->w_off[2], scale_at(sc, g->scale_code, g->s_off[2]), g->scale_code,
                        zp ? zp + g->z_off[2] : NULL, H, I, bits, gs, act, r, wd);
            for (int64_t q = count[e]; q < count[e + 1]; ++q) {
                int64_t j = order[q];
                const float* hj = hbuf + j * I;
                double acc = 0.0;
                for (int64_t k = 0; k < I; ++k) acc += (double)wd[k] * (double)hj[k];
                float y = round_act((float)acc, act);
                float w = load_val(rw, g->w_code, w_index ? w_index[j] : j);
                volatile float c = y * w;          /* one fp32 rounding, never fused */
                float cv = c;
                if (w_round) cv = round_act(cv, act);
                ybuf[j * H + r] = cv;
            }
        }
        free(wd);
    }
    /* Phase 3: each token's contributions summed in ascending expert id, then slot. */
    for (int64_t t = 0; t < T; ++t) {
        int64_t idx[64];
        int64_t kk = K < 64 ? K : 64;
        for (int64_t k = 0; k < kk; ++k) idx[k] = t * K + k;
        for (int64_t a = 1; a < kk; ++a) {           /* stable insertion sort by expert id */
            int64_t v = idx[a], b = a - 1;
            while (b >= 0 && eidx[idx[b]] > eidx[v]) { idx[b + 1] = idx[b]; --b; }
            idx[b + 1] = v;
        }
        for (int64_t c = 0; c < H; ++c) {
            float acc = 0.0f;
            for (int64_t k = 0; k < kk; ++k) {
                volatile float s = acc + ybuf[idx[k] * H + c];
                acc = s;
            }
            out[t * out_stride + c] = acc;
        }
    }
    if (h_out)
        for (int64_t j = 0; j < n; ++j)
            for (int64_t r = 0; r < I; ++r) store_val(h_out, act, j * I + r, hbuf[j * I + r]);
    if (y_out) memcpy(y_out, ybuf, sizeof(float) * (size_t)(n * H));
    free(count); free(order); free(xf); free(hbuf); free(ybuf); free(live);
    return K > 64 ? -4 : 0;
}

/* -------------------------------------------------------------------------------------- */
/* FP8 / FP4 block-scaled dequant and the fused GEMV                                        */
/* -------------------------------------------------------------------------------------- */

/* w [rows, cols] e4m3; scale [srows, scols] in scale_code (fp32 / bf16 / e8m0); out bf16. */
int vyo_fp8_dequant(const uint8_t* w, int64_t rows, int64_t cols, const void* scale,
                    int scale_code, int64_t srows, int64_t scols, uint16_t* out) {
    if (srows <= 0 || scols <= 0 || rows % srows || cols % scols) return -1;
    const int64_t bo = rows / srows, bi = cols / scols;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) {
            float s = load_val(scale, scale_code, (r / bo) * scols + c / bi);
            volatile float p = vyo_e4m3_to_f32(w[r * cols + c]) * s;
            out[r * cols + c] = vyo_f32_to_bf16(p);
        }
    return 0;
}

/* w [rows, cols/2] bytes, two e2m1 per byte, low nibble = even column; scale [rows, cols/gs]
 * e4m3; out [rows, cols] bf16. */
int vyo_fp4_dequant(const uint8_t* w, int64_t rows, int64_t cols, const uint8_t* scale,
                    int gs, uint16_t* out) {
    if (gs <= 0 || cols % gs || cols % 2) return -1;
    const int64_t groups = cols / gs;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) {
            uint8_t b = w[r * (cols / 2) + c / 2];
            uint32_t nib = (c & 1) ? (b >> 4) : (b & 15u);
            float s = vyo_e4m3_to_f32(scale[r * groups + c / gs]);
            volatile float p = e2m1_to_f32(nib) * s;
            out[r * cols + c] = vyo_f32_to_bf16(p);
        }
    return 0;
}

/* out[T, N] bf16 = x[T, K] (bf16) times the dequantised W[N, K]^T, summed in double and
 * rounded once.  kind 0 = fp8 (scale_code, srows, scols as vyo_fp8_dequant), kind 1 = fp4
 * (e4m3 scale per `gs`). */
int vyo_fp_gemv(int kind, const uint8_t* w, int64_t N, int64_t Kd, const void* scale,
                int scale_code, int64_t srows, int64_t scols, int gs, const uint16_t* x,
                int64_t T, uint16_t* out, int32_t n_threads) {
    if (kind == 0 && (srows <= 0 || scols <= 0 || N % srows || Kd % scols)) return -1;
    if (kind == 1 && (gs <= 0 || Kd % gs || Kd % 2)) return -1;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
    float* xf = (float*)malloc(sizeof(float) * (size_t)(T * Kd));
    if (!xf) return -2;
    for (int64_t i = 0; i < T * Kd; ++i) xf[i] = bf16_to_f32(x[i]);
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)Kd);
#pragma omp for schedule(dynamic, 16)
        for (int64_t n = 0; n < N; ++n) {
            for (int64_t c = 0; c < Kd; ++c) {
                float p;
                if (kind == 0) {
                    const int64_t bo = N / srows, bi = Kd / scols;
                    p = vyo_e4m3_to_f32(w[n * Kd + c]) *
                        load_val(scale, scale_code, (n / bo) * scols + c / bi);
                } else {
                    uint8_t b = w[n * (Kd / 2) + c / 2];
                    p = e2m1_to_f32((c & 1) ? (b >> 4) : (b & 15u)) *
                        vyo_e4m3_to_f32(((const uint8_t*)scale)[n * (Kd / gs) + c / gs]);
                }
                row[c] = bf16_to_f32(vyo_f32_to_bf16(p));
            }
            for (int64_t t = 0; t < T; ++t) {
                double acc = 0.0;
                const float* xt = xf + t * Kd;
                for (int64_t c = 0; c < Kd; ++c) acc += (double)row[c] * (double)xt[c];
                out[t * N + n] = vyo_f32_to_bf16((float)acc);
            }
        }
        free(row);
    }
    free(xf);
    return 0;
}
