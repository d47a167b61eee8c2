/*
 * moe_oracle.c -- CPU restatement of PocketLM's MoE expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the sm_100a
 * kernels in pocketlm_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product path never does.
 *
 * Every function restates one reference routine (paths are relative to the
 * PocketLM project root).  The floating-point operation order of the
 * reference is kept on purpose (block-of-128 partial sums in fp32, then the
 * block scale; SwiGLU as g / (1 + exp(-g)) * u), so that, compiled with
 * -ffp-contract=off, the results are bit-identical to the reference's own
 * scalar kernels.  tests/test_oracle_vs_reference.py checks that claim
 * against the reference compiled from source into oracle/_ref/.
 *
 * Conventions (mirroring the reference C ABI): every exported function
 * returns 0 on success and a small nonzero code on bad arguments; pointer
 * tables are arrays of uint64_t host addresses, one per expert.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_BLOCK 128

/* ------------------------------------------------------------------------ */
/* Scalar formats                                                            */
/* ------------------------------------------------------------------------ */

static float bits_to_f32(uint32_t bits) {
    float value;
    memcpy(&value, &bits, sizeof value);
    return value;
}

static uint32_t f32_to_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    return bits;
}

/* e4m3fn byte -> float.  `nan_is_zero` selects the two behaviours the
 * reference has for the all-ones codes 0x7F/0xFF:
 *   fp8_linear.cpp:19-36       (linear / MLP kernels)  -> +0.0f
 *   fp8_dequant.cpp:10-30      (dequant kernels)       -> quiet NaN       */
static float e4m3_to_f32(uint8_t code, int nan_is_zero) {
    const int negative = (code & 0x80u) != 0;
    const int exponent = (code >> 3) & 0xF;
    const int mantissa = code & 0x7;
    float magnitude;
    if (exponent == 0xF && mantissa == 0x7) {
        if (nan_is_zero) {
            return 0.0f;
        }
        /* the reference builds this exact NaN payload (fp8_dequant.cpp:22-27);
         * it survives an F16C conversion as 0x7F80 / 0xFF80 */
        return bits_to_f32(negative ? 0xFFF00000u : 0x7FF00000u);
    }
    if (exponent == 0) {
        /* subnormal: mantissa * 2^-9 */
        magnitude = ldexpf((float)mantissa, -9);
    } else {
        magnitude = ldexpf(8.0f + (float)mantissa, exponent - 10);
    }
    return negative ? -magnitude : magnitude;
}

static float g_e4m3_zero_nan[256];
static float g_e4m3_keep_nan[256];
static int g_tables_ready = 0;

static void build_tables(void) {
    if (g_tables_ready) {
        return;
    }
    for (int code = 0; code < 256; ++code) {
        g_e4m3_zero_nan[code] = e4m3_to_f32((uint8_t)code, 1);
        g_e4m3_keep_nan[code] = e4m3_to_f32((uint8_t)code, 0);
    }
    g_tables_ready = 1;
}

/* float -> bf16, round-to-nearest-even; NaN -> 0xFFFF.
 * fp8_dequant.cpp:108-117 */
static uint16_t f32_to_bf16_rne(float value) {
    if (isnan(value)) {
        return 0xFFFFu;
    }
    const uint32_t bits = f32_to_bits(value);
    const uint32_t keep_lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7FFFu + keep_lsb) >> 16);
}

static float bf16_to_f32(uint16_t value) {
    return bits_to_f32((uint32_t)value << 16);
}

/* IEEE binary16 <-> float, round-to-nearest-even.  Same results as the F16C
 * conversions the reference uses (fp8_dequant.cpp:81-106) and as the
 * hand-written ones in q4_dequant.cpp:10-90. */
static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exponent = (h >> 10) & 0x1Fu;
    uint32_t mantissa = h & 0x3FFu;
    if (exponent == 0x1Fu) {
        return bits_to_f32(sign | 0x7F800000u | (mantissa << 13));
    }
    if (exponent == 0) {
        /* zero or subnormal: mantissa * 2^-24, exact in float */
        const float magnitude = ldexpf((float)mantissa, -24);
        return sign ? -magnitude : magnitude;
    }
    return bits_to_f32(sign | ((exponent + 112u) << 23) | (mantissa << 13));
}

static uint16_t f32_to_f16_rne(float value) {
    const uint32_t bits = f32_to_bits(value);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    const uint32_t abs_bits = bits & 0x7FFFFFFFu;
    if (abs_bits > 0x7F800000u) {
        /* NaN: keep it quiet, keep the top payload bits */
        return (uint16_t)(sign | 0x7E00u | ((abs_bits >> 13) & 0x3FFu));
    }
    if (abs_bits >= 0x477FF000u) {
        /* >= 65520 rounds to infinity */
        return (uint16_t)(sign | 0x7C00u);
    }
    if (abs_bits < 0x38800000u) {
        /* result is subnormal or zero: scale to units of 2^-24 and round */
        const float magnitude = bits_to_f32(abs_bits);
        const float units = magnitude * 16777216.0f; /* exact: power of two */
        float rounded = nearbyintf(units);            /* default mode = RNE */
        return (uint16_t)(sign | (uint16_t)rounded);
    }
    /* normal range: rebias and round the 13 dropped bits to nearest even */
    uint32_t half = ((abs_bits - 0x38000000u) >> 13);
    const uint32_t dropped = abs_bits & 0x1FFFu;
    if (dropped > 0x1000u || (dropped == 0x1000u && (half & 1u))) {
        half += 1u; /* a carry into the exponent is the correct result */
    }
    return (uint16_t)(sign | half);
}

/* ------------------------------------------------------------------------ */
/* Block-scaled FP8 dot products                                             */
/* ------------------------------------------------------------------------ */

/* One output element of a 128x128 block-scaled FP8 linear, in the order the
 * reference accumulates it (fp8_linear.cpp:100-113): the 128 products of a
 * column block are summed left to right in fp32, the block sum is scaled by
 * scale_inv[row/128][block] and added to the running total. */
static float block_scaled_dot(const float* x, const uint8_t* w_row, const float* scale_row,
                              int64_t cols, int64_t scale_cols) {
    float total = 0.0f;
    for (int64_t block = 0; block < scale_cols; ++block) {
        const int64_t first = block * ORC_BLOCK;
        const int64_t last = first + ORC_BLOCK < cols ? first + ORC_BLOCK : cols;
        float partial = 0.0f;
        for (int64_t c = first; c < last; ++c) {
            const float product = x[c] * g_e4m3_zero_nan[w_row[c]];
            partial = partial + product;
        }
        const float scaled = partial * scale_row[block];
        total = total + scaled;
    }
    return total;
}

/* SwiGLU as the reference writes it (fp8_linear.cpp:333-334). */
static float swiglu(float gate, float up) {
    const float silu = gate / (1.0f + expf(-gate));
    return silu * up;
}

static int scale_cols_ok(int64_t cols, int64_t scale_cols) {
    return scale_cols == (cols + ORC_BLOCK - 1) / ORC_BLOCK;
}

/* fp8_e4m3_block_linear_f32, fp8_linear.cpp:50-117 */
int orc_fp8_linear_f32(const uint8_t* w, const float* scale_inv, const float* x, float* out,
                       int64_t batch, int64_t out_rows, int64_t in_cols, int64_t scale_cols) {
    if (!w || !scale_inv || !x || !out) return -1;
    if (batch <= 0 || out_rows <= 0 || in_cols <= 0 || scale_cols <= 0) return -2;
    build_tables();
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t r = 0; r < out_rows; ++r) {
            out[b * out_rows + r] = block_scaled_dot(x + b * in_cols, w + r * in_cols,
                                                     scale_inv + (r / ORC_BLOCK) * scale_cols,
                                                     in_cols, scale_cols);
        }
    }
    return 0;
}

/* fp8_e4m3_block_dual_linear_f32, fp8_linear.cpp:119-210 */
int orc_fp8_dual_linear_f32(const uint8_t* wa, const float* sa, const uint8_t* wb, const float* sb,
                            const float* x, float* out_a, float* out_b, int64_t batch,
                            int64_t out_rows, int64_t in_cols, int64_t scale_cols) {
    int code = orc_fp8_linear_f32(wa, sa, x, out_a, batch, out_rows, in_cols, scale_cols);
    if (code != 0) return code;
    return orc_fp8_linear_f32(wb, sb, x, out_b, batch, out_rows, in_cols, scale_cols);
}

/* The expert MLP of one token: act[i] = swiglu(gate_i . x, up_i . x).
 * fp8_linear.cpp:309-336 */
static void expert_activation(const float* x, const uint8_t* gate, const float* gate_s,
                              const uint8_t* up, const float* up_s, float* act,
                              int64_t inter, int64_t hidden, int64_t gate_scale_cols) {
    for (int64_t i = 0; i < inter; ++i) {
        const float* gs_row = gate_s + (i / ORC_BLOCK) * gate_scale_cols;
        const float* us_row = up_s + (i / ORC_BLOCK) * gate_scale_cols;
        const float g = block_scaled_dot(x, gate + i * hidden, gs_row, hidden, gate_scale_cols);
        const float u = block_scaled_dot(x, up + i * hidden, us_row, hidden, gate_scale_cols);
        act[i] = swiglu(g, u);
    }
}

/* fp8_e4m3_block_mlp_f32, fp8_linear.cpp:212-362 (non-reuse branch; the
 * batch-reuse branch at :248-307 has the same per-element order). */
int orc_fp8_mlp_f32(const uint8_t* gate, const float* gate_s, const uint8_t* up, const float* up_s,
                    const uint8_t* down, const float* down_s, const float* x, float* out,
                    int64_t batch, int64_t inter, int64_t hidden, int64_t gate_scale_cols,
                    int64_t down_scale_cols) {
    if (!gate || !gate_s || !up || !up_s || !down || !down_s || !x || !out) return -1;
    if (batch <= 0 || inter <= 0 || hidden <= 0 || gate_scale_cols <= 0 || down_scale_cols <= 0)
        return -2;
    build_tables();
    float* act = (float*)malloc((size_t)(batch * inter) * sizeof(float));
    if (!act) return -3;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t i = 0; i < inter; ++i) {
            const float* xb = x + b * hidden;
            const float g = block_scaled_dot(xb, gate + i * hidden,
                                             gate_s + (i / ORC_BLOCK) * gate_scale_cols, hidden,
                                             gate_scale_cols);
            const float u = block_scaled_dot(xb, up + i * hidden,
                                             up_s + (i / ORC_BLOCK) * gate_scale_cols, hidden,
                                             gate_scale_cols);
            act[b * inter + i] = swiglu(g, u);
        }
    }
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t h = 0; h < hidden; ++h) {
            out[b * hidden + h] = block_scaled_dot(act + b * inter, down + h * inter,
                                                   down_s + (h / ORC_BLOCK) * down_scale_cols,
                                                   inter, down_scale_cols);
        }
    }
    free(act);
    return 0;
}

/* Pointer-table access: table[e] holds a host address (fp8_linear.cpp:365-370). */
#define ORC_PTR(type, table, e) ((const type*)(uintptr_t)((table)[(e)]))

typedef struct {
    const uint64_t *gate, *gate_s, *up, *up_s, *down, *down_s;
} orc_tables;

static int tables_ok(const orc_tables* t) {
    return t->gate && t->gate_s && t->up && t->up_s && t->down && t->down_s;
}

static int expert_present(const orc_tables* t, int64_t e) {
    return t->gate[e] && t->gate_s[e] && t->up[e] && t->up_s[e];
}

/* Per-expert activations act[e][b][:] for every (expert, row) the `active`
 * predicate selects; rows not selected are left untouched. */
static void many_activations(const orc_tables* t, const float* x, float* act, int64_t experts,
                             int64_t batch, int64_t inter, int64_t hidden, int64_t gsc,
                             const float* row_weights /* [E,B] or NULL */) {
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t e = 0; e < experts; ++e) {
        for (int64_t b = 0; b < batch; ++b) {
            float* dst = act + (e * batch + b) * inter;
            if (row_weights && row_weights[e * batch + b] == 0.0f) continue;
            if (!expert_present(t, e)) {
                memset(dst, 0, (size_t)inter * sizeof(float));
                continue;
            }
            expert_activation(x + b * hidden, ORC_PTR(uint8_t, t->gate, e),
                              ORC_PTR(float, t->gate_s, e), ORC_PTR(uint8_t, t->up, e),
                              ORC_PTR(float, t->up_s, e), dst, inter, hidden, gsc);
        }
    }
}

static float expert_down_row(const orc_tables* t, int64_t e, const float* act_row, int64_t h,
                             int64_t inter, int64_t dsc) {
    const uint8_t* down = ORC_PTR(uint8_t, t->down, e);
    const float* down_s = ORC_PTR(float, t->down_s, e);
    return block_scaled_dot(act_row, down + h * inter, down_s + (h / ORC_BLOCK) * dsc, inter, dsc);
}

/* fp8_e4m3_block_mlp_many_f32, fp8_linear.cpp:364-473: out[E,B,H]. */
int orc_fp8_mlp_many_f32(const uint64_t* gp, const uint64_t* gsp, const uint64_t* upp,
                         const uint64_t* usp, const uint64_t* dp, const uint64_t* dsp,
                         const float* x, float* out, int64_t experts, int64_t batch,
                         int64_t inter, int64_t hidden, int64_t gsc, int64_t dsc) {
    orc_tables t = {gp, gsp, upp, usp, dp, dsp};
    if (!tables_ok(&t) || !x || !out) return -1;
    if (experts <= 0 || batch <= 0 || inter <= 0 || hidden <= 0 || gsc <= 0 || dsc <= 0) return -2;
    build_tables();
    float* act = (float*)malloc((size_t)(experts * batch * inter) * sizeof(float));
    if (!act) return -3;
    many_activations(&t, x, act, experts, batch, inter, hidden, gsc, NULL);
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t e = 0; e < experts; ++e) {
        for (int64_t b = 0; b < batch; ++b) {
            for (int64_t h = 0; h < hidden; ++h) {
                /* the reference skips (leaves unwritten) absent experts here */
                if (!t.down[e] || !t.down_s[e]) continue;
                out[(e * batch + b) * hidden + h] =
                    expert_down_row(&t, e, act + (e * batch + b) * inter, h, inter, dsc);
            }
        }
    }
    free(act);
    return 0;
}

/* fp8_e4m3_block_mlp_many_weighted_f32, fp8_linear.cpp:475-589:
 * out[b,h] = sum_e route[e] * y_e[b,h], experts in table order. */
int orc_fp8_mlp_many_weighted_f32(const uint64_t* gp, const uint64_t* gsp, const uint64_t* upp,
                                  const uint64_t* usp, const uint64_t* dp, const uint64_t* dsp,
                                  const float* x, const float* route, float* out, int64_t experts,
                                  int64_t batch, int64_t inter, int64_t hidden, int64_t gsc,
                                  int64_t dsc) {
    orc_tables t = {gp, gsp, upp, usp, dp, dsp};
    if (!tables_ok(&t) || !x || !route || !out) return -1;
    if (experts <= 0 || batch <= 0 || inter <= 0 || hidden <= 0 || gsc <= 0 || dsc <= 0) return -2;
    build_tables();
    float* act = (float*)malloc((size_t)(experts * batch * inter) * sizeof(float));
    if (!act) return -3;
    many_activations(&t, x, act, experts, batch, inter, hidden, gsc, NULL);
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < batch * hidden; ++idx) {
        const int64_t b = idx / hidden, h = idx % hidden;
        float routed = 0.0f;
        for (int64_t e = 0; e < experts; ++e) {
            if (!t.down[e] || !t.down_s[e]) continue;
            const float y = expert_down_row(&t, e, act + (e * batch + b) * inter, h, inter, dsc);
            const float contribution = route[e] * y;
            routed = routed + contribution;
        }
        out[idx] = routed;
    }
    free(act);
    return 0;
}

/* fp8_e4m3_block_mlp_many_row_weighted_f32, fp8_linear.cpp:591-831:
 * route is [E,B]; zero weights skip the (expert,row) work entirely. */
int orc_fp8_mlp_many_row_weighted_f32(const uint64_t* gp, const uint64_t* gsp, const uint64_t* upp,
                                      const uint64_t* usp, const uint64_t* dp, const uint64_t* dsp,
                                      const float* x, const float* route, float* out,
                                      int64_t experts, int64_t batch, int64_t inter,
                                      int64_t hidden, int64_t gsc, int64_t dsc) {
    orc_tables t = {gp, gsp, upp, usp, dp, dsp};
    if (!tables_ok(&t) || !x || !route || !out) return -1;
    if (experts <= 0 || batch <= 0 || inter <= 0 || hidden <= 0 || gsc <= 0 || dsc <= 0) return -2;
    build_tables();
    float* act = (float*)malloc((size_t)(experts * batch * inter) * sizeof(float));
    if (!act) return -3;
    many_activations(&t, x, act, experts, batch, inter, hidden, gsc, route);
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < batch * hidden; ++idx) {
        const int64_t b = idx / hidden, h = idx % hidden;
        float routed = 0.0f;
        for (int64_t e = 0; e < experts; ++e) {
            const float weight = route[e * batch + b];
            if (weight == 0.0f) continue;
            if (!t.down[e] || !t.down_s[e]) continue;
            const float y = expert_down_row(&t, e, act + (e * batch + b) * inter, h, inter, dsc);
            const float contribution = weight * y;
            routed = routed + contribution;
        }
        out[idx] = routed;
    }
    free(act);
    return 0;
}

/* fp8_e4m3_block_mlp_many_pair_weighted_f32, fp8_linear.cpp:833-980:
 * (item, row, weight) triples; out[b] sums the pairs of row b in pair order. */
int orc_fp8_mlp_many_pair_weighted_f32(const uint64_t* gp, const uint64_t* gsp, const uint64_t* upp,
                                       const uint64_t* usp, const uint64_t* dp, const uint64_t* dsp,
                                       const float* x, const int64_t* pair_item,
                                       const int64_t* pair_row, const float* pair_w, float* out,
                                       int64_t experts, int64_t pairs, int64_t batch, int64_t inter,
                                       int64_t hidden, int64_t gsc, int64_t dsc) {
    orc_tables t = {gp, gsp, upp, usp, dp, dsp};
    if (!tables_ok(&t) || !x || !pair_item || !pair_row || !pair_w || !out) return -1;
    if (experts <= 0 || pairs < 0 || batch <= 0 || inter <= 0 || hidden <= 0 || gsc <= 0 ||
        dsc <= 0)
        return -2;
    memset(out, 0, (size_t)(batch * hidden) * sizeof(float));
    if (pairs == 0) return 0;
    for (int64_t p = 0; p < pairs; ++p) {
        if (pair_item[p] < 0 || pair_item[p] >= experts || pair_row[p] < 0 || pair_row[p] >= batch)
            return -4;
    }
    build_tables();
    float* act = (float*)malloc((size_t)(pairs * inter) * sizeof(float));
    float* pair_out = (float*)malloc((size_t)(pairs * hidden) * sizeof(float));
    if (!act || !pair_out) {
        free(act);
        free(pair_out);
        return -3;
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t p = 0; p < pairs; ++p) {
        const int64_t e = pair_item[p];
        if (!expert_present(&t, e)) {
            memset(act + p * inter, 0, (size_t)inter * sizeof(float));
            continue;
        }
        expert_activation(x + pair_row[p] * hidden, ORC_PTR(uint8_t, t.gate, e),
                          ORC_PTR(float, t.gate_s, e), ORC_PTR(uint8_t, t.up, e),
                          ORC_PTR(float, t.up_s, e), act + p * inter, inter, hidden, gsc);
    }
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t p = 0; p < pairs; ++p) {
        for (int64_t h = 0; h < hidden; ++h) {
            const int64_t e = pair_item[p];
            pair_out[p * hidden + h] = (!t.down[e] || !t.down_s[e])
                                           ? 0.0f
                                           : expert_down_row(&t, e, act + p * inter, h, inter, dsc);
        }
    }
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < batch * hidden; ++idx) {
        const int64_t b = idx / hidden, h = idx % hidden;
        float routed = 0.0f;
        for (int64_t p = 0; p < pairs; ++p) {
            if (pair_row[p] != b) continue;
            const float contribution = pair_w[p] * pair_out[p * hidden + h];
            routed = routed + contribution;
        }
        out[idx] = routed;
    }
    free(act);
    free(pair_out);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Dequantisation                                                            */
/* ------------------------------------------------------------------------ */

/* fp8_e4m3_dequant_to_fp16 / _to_bf16, fp8_dequant.cpp:119-204:
 * out = round(lut[w] * scale) with NaN codes decoding to NaN. */
int orc_fp8_dequant(const uint8_t* w, const float* scale_inv, uint16_t* out, int64_t rows,
                    int64_t cols, int64_t scale_cols, int to_bf16) {
    if (!w || !scale_inv || !out) return -1;
    if (rows <= 0 || cols <= 0 || scale_cols <= 0) return -2;
    if (!scale_cols_ok(cols, scale_cols)) return -3;
    build_tables();
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            const float scale = scale_inv[(r / ORC_BLOCK) * scale_cols + c / ORC_BLOCK];
            const float value = g_e4m3_keep_nan[w[r * cols + c]] * scale;
            out[r * cols + c] = to_bf16 ? f32_to_bf16_rne(value) : f32_to_f16_rne(value);
        }
    }
    return 0;
}

/* Signed int4 at flat index `i`: even index = low nibble, codes >= 8 are
 * negative.  q4_dequant.cpp:120-128 (packing: q4_quantize.py:21-45). */
static int q4_code(const uint8_t* packed, int64_t i) {
    const uint8_t byte = packed[i >> 1];
    const int nibble = (i & 1) ? (byte >> 4) : (byte & 0xF);
    return nibble >= 8 ? nibble - 16 : nibble;
}

/* q4_dequant_to_fp16, q4_dequant.cpp:154-208: out = f16(q * scale[channel]). */
int orc_q4_dequant_to_fp16(const uint8_t* packed, const uint16_t* scales, uint16_t* out,
                           int64_t channels, int64_t channel_size) {
    if (!packed || !scales || !out) return 1;
    if (channels <= 0 || channel_size <= 0) return 2;
#pragma omp parallel for schedule(static)
    for (int64_t ch = 0; ch < channels; ++ch) {
        const float scale = f16_to_f32(scales[ch]);
        for (int64_t k = 0; k < channel_size; ++k) {
            const int64_t i = ch * channel_size + k;
            out[i] = f32_to_f16_rne((float)q4_code(packed, i) * scale);
        }
    }
    return 0;
}

/* Scalar Q4 row dot, q4_dequant.cpp:288-303: sum of (q * scale) * x[i]. */
static float q4_row_dot(const uint8_t* packed, const uint16_t* scales, int64_t row,
                        int64_t row_size, const float* x) {
    const float scale = f16_to_f32(scales[row]);
    float sum = 0.0f;
    for (int64_t k = 0; k < row_size; ++k) {
        const float w = (float)q4_code(packed, row * row_size + k) * scale;
        const float product = w * x[k];
        sum = sum + product;
    }
    return sum;
}

/* q4_moe_selected_forward_u16, q4_dequant.cpp:357-476: one fp16 token,
 * selected experts in table order, fp32 combine, fp16 output. */
int orc_q4_moe_selected_forward(const uint16_t* x_f16, const uint64_t* gate_p, const uint64_t* gate_s,
                                const uint64_t* up_p, const uint64_t* up_s, const uint64_t* down_p,
                                const uint64_t* down_s, const float* route, uint16_t* out_f16,
                                int64_t hidden, int64_t inter, int64_t selected) {
    if (!x_f16 || !gate_p || !gate_s || !up_p || !up_s || !down_p || !down_s || !route || !out_f16 ||
        hidden <= 0 || inter <= 0 || selected <= 0)
        return 1;
    for (int64_t e = 0; e < selected; ++e) {
        if (!gate_p[e] || !gate_s[e] || !up_p[e] || !up_s[e] || !down_p[e] || !down_s[e]) return 3;
    }
    float* x = (float*)malloc((size_t)hidden * sizeof(float));
    float* combined = (float*)calloc((size_t)hidden, sizeof(float));
    float* act = (float*)malloc((size_t)inter * sizeof(float));
    if (!x || !combined || !act) {
        free(x);
        free(combined);
        free(act);
        return 2;
    }
    for (int64_t k = 0; k < hidden; ++k) x[k] = f16_to_f32(x_f16[k]);
    for (int64_t e = 0; e < selected; ++e) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < inter; ++i) {
            const float g = q4_row_dot(ORC_PTR(uint8_t, gate_p, e), ORC_PTR(uint16_t, gate_s, e), i,
                                       hidden, x);
            const float u = q4_row_dot(ORC_PTR(uint8_t, up_p, e), ORC_PTR(uint16_t, up_s, e), i,
                                       hidden, x);
            act[i] = swiglu(g, u);
        }
#pragma omp parallel for schedule(static)
        for (int64_t h = 0; h < hidden; ++h) {
            const float d = q4_row_dot(ORC_PTR(uint8_t, down_p, e), ORC_PTR(uint16_t, down_s, e), h,
                                       inter, act);
            combined[h] = combined[h] + route[e] * d;
        }
    }
    for (int64_t h = 0; h < hidden; ++h) out_f16[h] = f32_to_f16_rne(combined[h]);
    free(x);
    free(combined);
    free(act);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* row8 packed GEMV and dense 16-bit experts                                 */
/* ------------------------------------------------------------------------ */

static float u16_to_f32(uint16_t v, int dtype_code) {
    return dtype_code == 1 ? bf16_to_f32(v) : f16_to_f32(v);
}

static uint16_t f32_to_u16(float v, int dtype_code) {
    if (dtype_code == 1) {
        /* fp16_moe.cpp:27-33 rounds to bf16 without a NaN special case */
        const uint32_t bits = f32_to_bits(v);
        return (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
    }
    return f32_to_f16_rne(v);
}

/* native_pack_u16_rows8, fp16_packed_gemv.cpp:52-77:
 * packed[block][col][lane] = weight[block*8+lane][col], zero padded. */
int orc_pack_rows8(const uint16_t* weight, uint16_t* packed, int64_t rows, int64_t cols) {
    if (!weight || !packed) return 1;
    if (rows < 0 || cols < 0) return 2;
    const int64_t blocks = (rows + 7) / 8;
    for (int64_t blk = 0; blk < blocks; ++blk) {
        for (int64_t c = 0; c < cols; ++c) {
            for (int64_t lane = 0; lane < 8; ++lane) {
                const int64_t r = blk * 8 + lane;
                packed[(blk * cols + c) * 8 + lane] = r < rows ? weight[r * cols + c] : 0;
            }
        }
    }
    return 0;
}

/* native_packed_gemv_rows8, fp16_packed_gemv.cpp:79-116: out[r] = sum_c x[c] * W[r,c]
 * accumulated column by column (the reference fuses multiply-add, so the
 * oracle matches it to within rounding, not bit for bit). */
int orc_packed_gemv_rows8(const uint16_t* x, const uint16_t* packed, float* out, int64_t rows,
                          int64_t cols, int dtype_code) {
    if (!x || !packed || !out) return 1;
    if (rows < 0 || cols < 0 || (dtype_code != 0 && dtype_code != 1)) return 2;
    const int64_t blocks = (rows + 7) / 8;
#pragma omp parallel for schedule(static)
    for (int64_t blk = 0; blk < blocks; ++blk) {
        double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int64_t c = 0; c < cols; ++c) {
            const double xc = u16_to_f32(x[c], dtype_code);
            for (int lane = 0; lane < 8; ++lane) {
                acc[lane] += xc * u16_to_f32(packed[(blk * cols + c) * 8 + lane], dtype_code);
            }
        }
        for (int lane = 0; lane < 8; ++lane) {
            const int64_t r = blk * 8 + lane;
            if (r < rows) out[r] = (float)acc[lane];
        }
    }
    return 0;
}

static double dot_u16(const float* x, const uint16_t* w, int64_t n, int dtype_code) {
    double acc = 0.0;
    for (int64_t k = 0; k < n; ++k) acc += (double)x[k] * u16_to_f32(w[k], dtype_code);
    return acc;
}

/* native_moe_selected_forward_u16, fp16_moe.cpp:199-267: per token, experts
 * already selected (weights stacked [S, rows, cols]), route [T, S]. */
int orc_moe_selected_forward_u16(const uint16_t* x, const uint16_t* gate, const uint16_t* up,
                                 const uint16_t* down, const float* route, uint16_t* out,
                                 int64_t seq_len, int64_t hidden, int64_t selected, int64_t inter,
                                 int dtype_code) {
    if (!x || !gate || !up || !down || !route || !out) return 1;
    if (seq_len <= 0 || hidden <= 0 || selected <= 0 || inter <= 0) return 2;
    if (dtype_code != 0 && dtype_code != 1) return 3;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < seq_len; ++t) {
        float* xf = (float*)malloc((size_t)hidden * sizeof(float));
        float* act = (float*)malloc((size_t)inter * sizeof(float));
        double* combined = (double*)calloc((size_t)hidden, sizeof(double));
        for (int64_t k = 0; k < hidden; ++k) xf[k] = u16_to_f32(x[t * hidden + k], dtype_code);
        for (int64_t s = 0; s < selected; ++s) {
            const uint16_t* g = gate + s * inter * hidden;
            const uint16_t* u = up + s * inter * hidden;
            const uint16_t* d = down + s * hidden * inter;
            for (int64_t i = 0; i < inter; ++i) {
                act[i] = swiglu((float)dot_u16(xf, g + i * hidden, hidden, dtype_code),
                                (float)dot_u16(xf, u + i * hidden, hidden, dtype_code));
            }
            const double w = route[t * selected + s];
            for (int64_t h = 0; h < hidden; ++h) {
                combined[h] += w * (float)dot_u16(act, d + h * inter, inter, dtype_code);
            }
        }
        for (int64_t h = 0; h < hidden; ++h) out[t * hidden + h] = f32_to_u16((float)combined[h], dtype_code);
        free(xf);
        free(act);
        free(combined);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Softmax router (Mixtral/Qwen style) and the expert-output combine         */
/* ------------------------------------------------------------------------ */

/* Top-k of `score` with ties to the lower id (ds_forward.cpp:931-943). */
static void topk_ids(const float* score, int64_t n, int64_t k, int64_t* ids) {
    for (int64_t j = 0; j < k; ++j) ids[j] = -1;
    for (int64_t j = 0; j < k; ++j) {
        int64_t best = -1;
        for (int64_t e = 0; e < n; ++e) {
            int taken = 0;
            for (int64_t q = 0; q < j; ++q) taken |= (ids[q] == e);
            if (taken) continue;
            if (best < 0 || score[e] > score[best]) best = e;
        }
        ids[j] = best;
    }
}

/* ds_router_topk_u16, ds_forward.cpp:879-955: fp32 logits from 16-bit
 * inputs, exp(s - max) with an fp64 denominator, top-k, fp64 renorm. */
int orc_router_softmax_topk_u16(const uint16_t* x, const uint16_t* w, int64_t hidden,
                                int64_t experts, int64_t k, int dtype_code, int64_t* out_ids,
                                float* out_w) {
    if (!x || !w || !out_ids || !out_w) return 1;
    if (hidden <= 0 || experts <= 0 || k <= 0 || k > experts) return 2;
    float* prob = (float*)malloc((size_t)experts * sizeof(float));
    if (!prob) return 3;
    for (int64_t e = 0; e < experts; ++e) {
        float logit = 0.0f;
        for (int64_t c = 0; c < hidden; ++c) {
            const float product = u16_to_f32(x[c], dtype_code) * u16_to_f32(w[e * hidden + c], dtype_code);
            logit = logit + product;
        }
        prob[e] = logit;
    }
    float top = prob[0];
    for (int64_t e = 1; e < experts; ++e) top = prob[e] > top ? prob[e] : top;
    double denom = 0.0;
    for (int64_t e = 0; e < experts; ++e) {
        prob[e] = expf(prob[e] - top);
        denom += (double)prob[e];
    }
    for (int64_t e = 0; e < experts; ++e) prob[e] = (float)((double)prob[e] / denom);
    topk_ids(prob, experts, k, out_ids);
    double picked = 0.0;
    for (int64_t j = 0; j < k; ++j) picked += (double)prob[out_ids[j]];
    if (picked <= 0.0) {
        free(prob);
        return 4;
    }
    for (int64_t j = 0; j < k; ++j) out_w[j] = (float)((double)prob[out_ids[j]] / picked);
    free(prob);
    return 0;
}

/* ds_moe_layer_forward_f32, ds_forward.cpp:337-367:
 * out[i] = sum_e route[e] * outputs[e][i], experts in order. */
int orc_combine_f32(const float* expert_outputs, const float* route, int64_t selected,
                    int64_t batch, int64_t hidden, float* out) {
    if (!expert_outputs || !route || !out) return 1;
    if (selected <= 0 || batch <= 0 || hidden <= 0) return 2;
    const int64_t width = batch * hidden;
    for (int64_t i = 0; i < width; ++i) {
        float acc = 0.0f;
        for (int64_t e = 0; e < selected; ++e) {
            const float contribution = route[e] * expert_outputs[e * width + i];
            acc = acc + contribution;
        }
        out[i] = acc;
    }
    return 0;
}

/* Exposed for the Python side of the oracle (tests of the scalar formats). */
void orc_f32_to_f16_array(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16_rne(in[i]);
}

void orc_e4m3_decode_array(const uint8_t* in, float* out, int64_t n, int nan_is_zero) {
    build_tables();
    for (int64_t i = 0; i < n; ++i) out[i] = nan_is_zero ? g_e4m3_zero_nan[in[i]] : g_e4m3_keep_nan[in[i]];
}
