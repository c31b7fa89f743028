/*
 * acfun_oracle.c — TEST INFRASTRUCTURE ONLY (see acfun_oracle.h).
 *
 * Plain C11, single-threaded, compiled with -ffp-contract=off so that every float
 * expression rounds exactly as written.  Reference citations are path:line inside the
 * hit-droid/Acfun tree.
 */
#include "acfun_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float fmaxf_ref(float a, float b) { return a > b ? a : b; }

/* ====================================================================== GEMM */

/* gemm_ref.cpp:43-63 (acfun_gemm_ref_epi): k-outer row update, zero A entries skipped,
 * bias added once after the reduction, then optional ReLU. */
void orc_gemm_f32(int M, int N, int K, const float* A, const float* B, float* C,
                  const float* bias, int act) {
    for (int i = 0; i < M; ++i) {
        const float* a = A + (size_t)i * K;
        float* c = C + (size_t)i * N;
        for (int j = 0; j < N; ++j) c[j] = 0.0f;
        for (int k = 0; k < K; ++k) {
            float av = a[k];
            if (av == 0.0f) continue;
            const float* b = B + (size_t)k * N;
            for (int j = 0; j < N; ++j) c[j] += av * b[j];
        }
        for (int j = 0; j < N; ++j) {
            float v = c[j];
            if (bias) v += bias[j];
            if (act && v < 0.0f) v = 0.0f;
            c[j] = v;
        }
    }
}

/* gemm_bf16_avx512.cpp:37-44: RNE by adding 0x7fff + lsb, NaN/Inf not special-cased. */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t rounding = 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)((x + rounding) >> 16);
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* gemm_bf16_avx512.cpp:88-114,171-232: both operands rounded to bf16, products exact in
 * fp32, accumulated in fp32.  (The reference's M%16/N%16 tails are pure fp32,
 * :161-168; the bf16 tolerance covers that difference.) */
void orc_gemm_bf16(int M, int N, int K, const float* A, const float* B, float* C) {
    float* Bb = (float*)malloc((size_t)K * N * sizeof(float));
    for (size_t t = 0; t < (size_t)K * N; ++t) Bb[t] = bf16_to_f32(orc_f32_to_bf16(B[t]));
    for (int i = 0; i < M; ++i) {
        float* c = C + (size_t)i * N;
        for (int j = 0; j < N; ++j) c[j] = 0.0f;
        for (int k = 0; k < K; ++k) {
            float av = bf16_to_f32(orc_f32_to_bf16(A[(size_t)i * K + k]));
            const float* b = Bb + (size_t)k * N;
            for (int j = 0; j < N; ++j) c[j] += av * b[j];
        }
    }
    free(Bb);
}

/* gemm_int8.cpp:11-25 (acfun_gemm_int8_ref_ld): exact u8 x s8 -> s32. */
void orc_gemm_int8(int M, int N, int K, const uint8_t* A, const int8_t* B, int32_t* C) {
    for (int i = 0; i < M; ++i) {
        int32_t* c = C + (size_t)i * N;
        for (int j = 0; j < N; ++j) c[j] = 0;
        for (int k = 0; k < K; ++k) {
            int32_t av = A[(size_t)i * K + k];
            if (av == 0) continue;
            const int8_t* b = B + (size_t)k * N;
            for (int j = 0; j < N; ++j) c[j] += av * (int32_t)b[j];
        }
    }
}

/* gemm_int8.cpp:53-67 (acfun_gemm_int8_epi_ref) and the mul-then-add of
 * gemm_int8_avx512.cpp:126-127: v = (float)acc * alpha[j]; v = v + beta[j]; ReLU. */
void orc_gemm_int8_epi(int M, int N, int K, const uint8_t* A, const int8_t* B, float* C,
                       const float* alpha, const float* beta, int act) {
    int32_t* acc = (int32_t*)malloc((size_t)N * sizeof(int32_t));
    for (int i = 0; i < M; ++i) {
        orc_gemm_int8(1, N, K, A + (size_t)i * K, B, acc);
        for (int j = 0; j < N; ++j) {
            float v = (float)acc[j] * alpha[j];
            v = v + beta[j];
            if (act && v < 0.0f) v = 0.0f;
            C[(size_t)i * N + j] = v;
        }
    }
    free(acc);
}

/* Requantising s8 x s8 GEMM.  No reference counterpart: the reference takes u8
 * activations and stops at fp32 (gemm_int8_avx512.cpp:364-377).  Definition used by the
 * BASELINE int8 GEMM config: exact int32 bias add, one RN int->float conversion, one RN
 * multiply by the per-column scale, optional ReLU, RNE to integer, saturate to s8. */
int8_t orc_requant_s8(int32_t acc, int32_t bias, float scale, int act) {
    int32_t s = (int32_t)((uint32_t)acc + (uint32_t)bias);   /* wrapping add, like the GPU */
    float v = (float)s * scale;
    if (act && !(v > 0.0f)) v = 0.0f;                         /* max(0, v); NaN -> 0 */
    float r = rintf(v);                                       /* RNE (default rounding mode) */
    if (r > 127.0f) r = 127.0f;
    if (r < -128.0f) r = -128.0f;
    if (r != r) r = 0.0f;
    return (int8_t)(int)r;
}

void orc_gemm_s8_requant(int M, int N, int K, const int8_t* A, const int8_t* B,
                         const int32_t* bias, const float* scale, int8_t* C, int act) {
    int32_t* acc = (int32_t*)malloc((size_t)N * sizeof(int32_t));
    for (int i = 0; i < M; ++i) {
        for (int j = 0; j < N; ++j) acc[j] = 0;
        for (int k = 0; k < K; ++k) {
            int32_t av = A[(size_t)i * K + k];
            const int8_t* b = B + (size_t)k * N;
            for (int j = 0; j < N; ++j) acc[j] += av * (int32_t)b[j];
        }
        for (int j = 0; j < N; ++j)
            C[(size_t)i * N + j] = orc_requant_s8(acc[j], bias ? bias[j] : 0, scale[j], act);
    }
    free(acc);
}

/* ============================================================ quantization */

/* int8_quantize_avx512.cpp:8-35 (rne=1: _mm512_cvtps_epi32 under the default MXCSR,
 * round-to-nearest-even) and int8_quantize.cpp:15-20 (rne=0: lroundf, ties away). */
void orc_quantize_u8(const float* in, uint8_t* out, size_t n, float inv_s, int zp, int rne) {
    for (size_t i = 0; i < n; ++i) {
        float t = in[i] * inv_s;
        int v = rne ? (int)rintf(t) : (int)lroundf(t);
        v += zp;
        out[i] = (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
    }
}

/* conv_int8.cpp:24-37: per-column symmetric scale, IEEE division, lroundf, clamp. */
void orc_quantize_weights(const float* w, int K, int N, float* scales, int8_t* wq) {
    for (int j = 0; j < N; ++j) {
        float maxa = 0.0f;
        for (int k = 0; k < K; ++k) maxa = fmaxf_ref(maxa, fabsf(w[(size_t)k * N + j]));
        float s = maxa / 127.0f;
        if (s <= 0.0f) s = 1.0f;
        scales[j] = s;
        for (int k = 0; k < K; ++k) {
            int v = (int)lroundf(w[(size_t)k * N + j] / s);
            if (v > 127) v = 127; else if (v < -128) v = -128;
            wq[(size_t)k * N + j] = (int8_t)v;
        }
    }
}

/* ======================================================= int8 convolution */

/* winograd_int8.cpp:54-70 — BT d BT^T on one 4x4 u8 block, int16 arithmetic. */
static void wi8_input_transform(const uint8_t d[16], int16_t dh[16]) {
    int16_t U[4][4];
    for (int l = 0; l < 4; ++l) {
        int16_t c0 = d[l], c1 = d[4 + l], c2 = d[8 + l], c3 = d[12 + l];
        U[0][l] = (int16_t)(c0 - c2);
        U[1][l] = (int16_t)(c1 + c2);
        U[2][l] = (int16_t)(-c1 + c2);
        U[3][l] = (int16_t)(-c1 + c3);
    }
    for (int i = 0; i < 4; ++i) {
        int16_t u0 = U[i][0], u1 = U[i][1], u2 = U[i][2], u3 = U[i][3];
        dh[i * 4 + 0] = (int16_t)(u0 - u2);
        dh[i * 4 + 1] = (int16_t)(u1 + u2);
        dh[i * 4 + 2] = (int16_t)(-u1 + u2);
        dh[i * 4 + 3] = (int16_t)(-u1 + u3);
    }
}

/* winograd_int8.cpp:74-90 — G~ g G~^T with G~ = 2G (integer, carries a x4 scale). */
static void wi8_filter_transform(const int8_t g[9], int16_t gh2[16]) {
    int16_t T[4][3];
    for (int y = 0; y < 3; ++y) {
        int16_t a = g[y], b = g[3 + y], c = g[6 + y];
        T[0][y] = (int16_t)(2 * a);
        T[1][y] = (int16_t)(a + b + c);
        T[2][y] = (int16_t)(a - b + c);
        T[3][y] = (int16_t)(2 * c);
    }
    for (int i = 0; i < 4; ++i) {
        int16_t t0 = T[i][0], t1 = T[i][1], t2 = T[i][2];
        gh2[i * 4 + 0] = (int16_t)(2 * t0);
        gh2[i * 4 + 1] = (int16_t)(t0 + t1 + t2);
        gh2[i * 4 + 2] = (int16_t)(t0 - t1 + t2);
        gh2[i * 4 + 3] = (int16_t)(2 * t2);
    }
}

/* winograd_int8.cpp:245-350 (+ tile :175-237, output :127-171), restated per tile.
 * The in-place quantiser is trunc(t + copysign(0.5, t)) for whole 16-channel groups
 * (:306-320) and lroundf for the Cin%16 tail channels (:321-325).  T4 accumulates in
 * int32 with wrap-around exactly like the vpmaddwd / vpaddd chain; the output transform
 * runs in int64 and converts with round-to-nearest; dequant is one fmaf with
 * wso = (s_in * 0.25f) * wscale[o]. */
void orc_winograd_int8(const float* input, int N, int H, int W, int Cin,
                       const int8_t* wq, const float* wscale, const float* bias, int Cout,
                       float s_in, float inv_s, float* output, int act) {
    const int OH = H, OW = W, tH = (OH + 1) / 2, tW = (OW + 1) / 2, ZP = 128;
    static const int AT[2][4] = {{1, 1, 1, 0}, {0, 1, -1, 1}};
    int16_t* gh2 = (int16_t*)malloc((size_t)16 * Cin * Cout * sizeof(int16_t));
    int32_t* Sgh = (int32_t*)calloc((size_t)16 * Cout, sizeof(int32_t));
    for (int c = 0; c < Cin; ++c)
        for (int o = 0; o < Cout; ++o) {
            int8_t g[9];
            int16_t t[16];
            for (int k = 0; k < 9; ++k) g[k] = wq[((size_t)k * Cin + c) * Cout + o];
            wi8_filter_transform(g, t);
            for (int ij = 0; ij < 16; ++ij) {
                gh2[((size_t)ij * Cin + c) * Cout + o] = t[ij];
                Sgh[(size_t)ij * Cout + o] += t[ij];
            }
        }
    const int Hp = H + 2, Wp = W + 2;
    uint8_t* pad = (uint8_t*)malloc((size_t)Hp * Wp * Cin);
    int16_t* dh = (int16_t*)malloc((size_t)16 * Cin * sizeof(int16_t));
    int32_t* T4 = (int32_t*)malloc((size_t)16 * Cout * sizeof(int32_t));
    const int cvec = Cin & ~15;
    for (int n = 0; n < N; ++n) {
        const float* x = input + (size_t)n * H * W * Cin;
        memset(pad, ZP, (size_t)Hp * Wp * Cin);
        for (int ih = 0; ih < H; ++ih)
            for (int iw = 0; iw < W; ++iw) {
                uint8_t* dst = pad + ((size_t)(ih + 1) * Wp + (iw + 1)) * Cin;
                const float* xr = x + ((size_t)ih * W + iw) * Cin;
                for (int c = 0; c < Cin; ++c) {
                    int v;
                    if (c < cvec) {
                        float t = xr[c] * inv_s;
                        float r = t + copysignf(0.5f, t);
                        float tr = truncf(r);
                        /* cvttps2dq: out-of-range -> INT_MIN; |t| stays far below 2^31 here */
                        v = (fabsf(tr) < 2147483648.0f) ? (int)tr : (int)0x80000000;
                        v += ZP;
                    } else {
                        v = (int)lroundf(xr[c] * inv_s) + ZP;
                    }
                    if (v < 0) v = 0; else if (v > 255) v = 255;
                    dst[c] = (uint8_t)v;
                }
            }
        float* yo = output + (size_t)n * OH * OW * Cout;
        for (int ty = 0; ty < tH; ++ty)
            for (int tx = 0; tx < tW; ++tx) {
                for (int c = 0; c < Cin; ++c) {
                    uint8_t blk[16];
                    int16_t t[16];
                    for (int k = 0; k < 4; ++k)
                        for (int l = 0; l < 4; ++l) {
                            int pr = 2 * ty + k, pc = 2 * tx + l;
                            blk[k * 4 + l] = (pr < Hp && pc < Wp)
                                ? pad[((size_t)pr * Wp + pc) * Cin + c] : (uint8_t)ZP;
                        }
                    wi8_input_transform(blk, t);
                    for (int ij = 0; ij < 16; ++ij) dh[(size_t)ij * Cin + c] = t[ij];
                }
                for (int ij = 0; ij < 16; ++ij)
                    for (int o = 0; o < Cout; ++o) {
                        uint32_t acc = 0;
                        for (int c = 0; c < Cin; ++c)
                            acc += (uint32_t)((int32_t)dh[(size_t)ij * Cin + c] *
                                              (int32_t)gh2[((size_t)ij * Cin + c) * Cout + o]);
                        if (ij == 5) acc -= (uint32_t)(512 * Sgh[(size_t)ij * Cout + o]);
                        T4[(size_t)ij * Cout + o] = (int32_t)acc;
                    }
                for (int e = 0; e < 4; ++e) {
                    int oh = 2 * ty + (e >> 1), ow = 2 * tx + (e & 1);
                    if (oh >= OH || ow >= OW) continue;
                    for (int o = 0; o < Cout; ++o) {
                        int64_t y = 0;
                        for (int ij = 0; ij < 16; ++ij) {
                            int s = AT[e >> 1][ij >> 2] * AT[e & 1][ij & 3];
                            y += (int64_t)s * (int64_t)T4[(size_t)ij * Cout + o];
                        }
                        float wso = (s_in * 0.25f) * wscale[o];
                        float v = fmaf((float)y, wso, bias ? bias[o] : 0.0f);
                        if (act == 1) v = fmaxf_ref(v, 0.0f);
                        yo[((size_t)oh * OW + ow) * Cout + o] = v;
                    }
                }
            }
    }
    free(gh2); free(Sgh); free(pad); free(dh); free(T4);
}

/* conv_int8_direct.cpp:20-59: every tap accumulated, out-of-bounds taps read zp=128,
 * epilogue mul-then-add. */
void orc_conv2d_int8_direct(const uint8_t* inQ, int N, int H, int W, int Cin,
                            const int8_t* wq, const float* alpha, const float* beta,
                            int KH, int KW, int Cout, int stride, int pad,
                            int OH, int OW, float* output, int act) {
    const int ZP = 128;
    for (int n = 0; n < N; ++n)
        for (int oh = 0; oh < OH; ++oh)
            for (int ow = 0; ow < OW; ++ow) {
                float* dst = output + (((size_t)n * OH + oh) * OW + ow) * Cout;
                for (int j = 0; j < Cout; ++j) {
                    int32_t acc = 0;
                    for (int kh = 0; kh < KH; ++kh) {
                        int ih = oh * stride - pad + kh;
                        for (int kw = 0; kw < KW; ++kw) {
                            int iw = ow * stride - pad + kw;
                            int ok = ih >= 0 && ih < H && iw >= 0 && iw < W;
                            const uint8_t* ip = inQ + (((size_t)n * H + (ok ? ih : 0)) * W + (ok ? iw : 0)) * Cin;
                            const int8_t* wp = wq + (size_t)((kh * KW + kw) * Cin) * Cout + j;
                            for (int ic = 0; ic < Cin; ++ic)
                                acc += (ok ? (int32_t)ip[ic] : ZP) * (int32_t)wp[(size_t)ic * Cout];
                        }
                    }
                    float v = (float)acc * alpha[j];
                    v = v + beta[j];
                    if (act && v < 0.0f) v = 0.0f;
                    dst[j] = v;
                }
            }
}

/* conv1x1_int8.cpp:21-36 */
void orc_conv1x1_int8(const uint8_t* inQ, int M, int K, int Cout, const int8_t* wq,
                      const float* alpha, const float* beta, float* output, int act) {
    orc_gemm_int8_epi(M, Cout, K, inQ, wq, output, alpha, beta, act);
}

int orc_conv2d_int8_route(const float* input, int N, int H, int W, int Cin,
                          int KH, int KW, int Cout, int stride, int pad) {
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (OH <= 0 || OW <= 0) return -1;
    size_t inN = (size_t)N * H * W * Cin;
    float maxa = 0.0f;
    for (size_t i = 0; i < inN; ++i) maxa = fmaxf_ref(maxa, fabsf(input[i]));
    if (maxa < 1e-12f) return 0;
    if (KH == 3 && KW == 3 && stride == 1 && pad == 1 && H >= 3 && W >= 3 && Cin >= 4 && Cout >= 4)
        return 1;
    int K = KH * KW * Cin;
    int zero_copy = (KH == 1 && KW == 1 && stride == 1 && pad == 0);
    if (K <= 64 && !zero_copy) return 2;
    if (zero_copy) return 3;
    return 4;
}

/* conv_int8.cpp:63-148 — the router: per-tensor max|x|, inv_s = 127/maxa, sa = maxa/127,
 * s_in ignored; Winograd route quantises inside; the others quantise with RNE
 * (AVX-512 host), then share alpha[j] = sa*ws[j], beta[j] = bias[j] - (alpha*128)*Sw[j]
 * with Sw a float sum (exact for these magnitudes). */
void orc_conv2d_int8(const float* input, int N, int H, int W, int Cin,
                     const int8_t* wq, const float* wscale, const float* bias,
                     int KH, int KW, int Cout, int stride, int pad,
                     float s_in, float* output, int act) {
    (void)s_in;
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (OH <= 0 || OW <= 0) return;
    int K = KH * KW * Cin;
    size_t M = (size_t)N * OH * OW;
    size_t inN = (size_t)N * H * W * Cin;
    float maxa = 0.0f;
    for (size_t i = 0; i < inN; ++i) maxa = fmaxf_ref(maxa, fabsf(input[i]));
    if (maxa < 1e-12f) { memset(output, 0, M * Cout * sizeof(float)); return; }
    const int ZP = 128;
    float inv_s = 127.0f / maxa;
    float sa = maxa / 127.0f;
    if (KH == 3 && KW == 3 && stride == 1 && pad == 1 && H >= 3 && W >= 3 && Cin >= 4 && Cout >= 4) {
        orc_winograd_int8(input, N, H, W, Cin, wq, wscale, bias, Cout, sa, inv_s, output, act);
        return;
    }
    uint8_t* inQ = (uint8_t*)malloc(inN ? inN : 1);
    orc_quantize_u8(input, inQ, inN, inv_s, ZP, 1);
    float* alpha = (float*)malloc((size_t)Cout * sizeof(float));
    float* beta = (float*)malloc((size_t)Cout * sizeof(float));
    for (int j = 0; j < Cout; ++j) {
        float Swj = 0.0f;
        for (int k = 0; k < K; ++k) Swj += (float)wq[(size_t)k * Cout + j];
        float a = sa * wscale[j];
        alpha[j] = a;
        float corr = a * (float)ZP;
        corr = corr * Swj;
        beta[j] = (bias ? bias[j] : 0.0f) - corr;
    }
    int zero_copy = (KH == 1 && KW == 1 && stride == 1 && pad == 0);
    if (K <= 64 && !zero_copy) {
        orc_conv2d_int8_direct(inQ, N, H, W, Cin, wq, alpha, beta, KH, KW, Cout, stride, pad,
                               OH, OW, output, act);
    } else {
        /* 1x1 zero-copy route and the im2col+GEMM-epi route (conv_int8.cpp:128-147) are the
         * same arithmetic as the direct route: exact integer correlation with zp padding
         * followed by the shared mul-then-add epilogue. */
        orc_conv2d_int8_direct(inQ, N, H, W, Cin, wq, alpha, beta, KH, KW, Cout, stride, pad,
                               OH, OW, output, act);
    }
    free(inQ); free(alpha); free(beta);
}

/* ====================================================== float convolution */

/* Naive direct convolution, accumulation kh -> kw -> ic per output, starting from the
 * bias, one rounding per multiply and per add.  Layouts: groups==1 -> [KH*KW*Cin][Cout]
 * (acfun.h:54-58); groups==Cin==Cout -> [C][KH][KW] (acfun.h:72-73); other groups ->
 * [g][KH*KW*Cin_per][Cout_per] (group_conv.cpp:137-139).  The depthwise and grouped-direct
 * routes go to their exact restatements below. */
static void conv_naive(const float* input, int N, int H, int W, int Cin,
                       const float* weight, const float* bias, int KH, int KW, int Cout,
                       int stride, int pad, int groups, float* output, int act) {
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    int Cin_p = Cin / groups, Cout_p = Cout / groups;
    for (int n = 0; n < N; ++n)
        for (int oh = 0; oh < OH; ++oh)
            for (int ow = 0; ow < OW; ++ow)
                for (int oc = 0; oc < Cout; ++oc) {
                    int g = oc / Cout_p, ocp = oc % Cout_p;
                    float s = bias ? bias[oc] : 0.0f;
                    for (int kh = 0; kh < KH; ++kh) {
                        int ih = oh * stride - pad + kh;
                        if (ih < 0 || ih >= H) continue;
                        for (int kw = 0; kw < KW; ++kw) {
                            int iw = ow * stride - pad + kw;
                            if (iw < 0 || iw >= W) continue;
                            const float* ip = input + (((size_t)n * H + ih) * W + iw) * Cin + (size_t)g * Cin_p;
                            for (int ic = 0; ic < Cin_p; ++ic) {
                                float wv = weight[(size_t)g * KH * KW * Cin_p * Cout_p +
                                                  ((size_t)(kh * KW + kw) * Cin_p + ic) * Cout_p + ocp];
                                s += ip[ic] * wv;
                            }
                        }
                    }
                    if (act && s < 0.0f) s = 0.0f;
                    output[(((size_t)n * OH + oh) * OW + ow) * Cout + oc] = s;
                }
}

void orc_conv2d(const float* input, int N, int H, int W, int Cin,
                const float* weight, const float* bias, int KH, int KW, int Cout,
                int stride, int pad, int groups, float* output, int act) {
    if (groups < 1) groups = 1;
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (OH <= 0 || OW <= 0) return;
    if (groups > 1 && groups == Cin && groups == Cout) {   /* layers.cpp:112-116 */
        orc_conv2d_dw(input, N, H, W, Cin, weight, bias, KH, KW, stride, pad, output, act);
        return;
    }
    if (groups > 1 && Cin / groups <= 64 && Cout / groups <= 128) {   /* layers.cpp:126-130 */
        orc_group_conv(input, N, H, W, Cin, weight, bias, KH, KW, Cout, stride, pad, groups,
                       output, act);
        return;
    }
    conv_naive(input, N, H, W, Cin, weight, bias, KH, KW, Cout, stride, pad, groups, output, act);
}

/* dw_avx512.cpp:20-74 (the route on an AVX-512 host, dw.cpp:47-58): per output channel the
 * accumulator starts at the bias and takes one fused multiply-add per tap, kh -> kw, a tap
 * outside the image contributing fma(0, w, acc); ReLU is max(acc, 0) (vmaxps: acc > 0 ? acc : 0). */
void orc_conv2d_dw(const float* input, int N, int H, int W, int C, const float* weight,
                   const float* bias, int KH, int KW, int stride, int pad, float* output, int act) {
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (OH <= 0 || OW <= 0 || KH <= 0 || KW <= 0) return;
    for (int n = 0; n < N; ++n)
        for (int oh = 0; oh < OH; ++oh)
            for (int ow = 0; ow < OW; ++ow)
                for (int c = 0; c < C; ++c) {
                    float acc = bias ? bias[c] : 0.0f;
                    for (int kh = 0; kh < KH; ++kh)
                        for (int kw = 0; kw < KW; ++kw) {
                            int ih = oh * stride - pad + kh, iw = ow * stride - pad + kw;
                            float v = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                                          ? input[(((size_t)n * H + ih) * W + iw) * C + c] : 0.0f;
                            acc = fmaf(v, weight[((size_t)c * KH + kh) * KW + kw], acc);
                        }
                    if (act == 1) acc = acc > 0.0f ? acc : 0.0f;
                    output[(((size_t)n * OH + oh) * OW + ow) * C + c] = acc;
                }
}

/* group_conv.cpp:62-79 dispatch on an AVX-512 host: Cout_per >= 16 -> group_conv_avx512.cpp
 * (every output channel, the masked tail included, one fma per (tap, input channel));
 * 8 <= Cout_per < 16 -> group_conv_avx2.cpp (whole 8-channel blocks with fma, the remaining
 * Cout_per % 8 channels in its scalar loop: mul, then add as written); narrower -> the scalar
 * kernel group_conv.cpp:16-55 (mul, then add).  Taps outside the image are skipped;
 * accumulation from the bias, kh -> kw -> ic.  Bit-exact against the compiled reference for
 * Cout_per a multiple of 8, >= 16 or < 8; for the AVX2 tail channels (Cout_per % 8 != 0 below
 * 16) the compiled reference's rounding depends on how the compiler translated that scalar loop
 * (measured: matches for Cin_per = 4, not for Cin_per = 5), so such shapes are pinned within
 * the fp32 tolerance only. */
void orc_group_conv(const float* input, int N, int H, int W, int Cin, const float* weight,
                    const float* bias, int KH, int KW, int Cout, int stride, int pad,
                    int groups, float* output, int act) {
    int Cin_p = Cin / groups, Cout_p = Cout / groups;
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (OH <= 0 || OW <= 0) return;
    const int fused_below = Cout_p >= 16 ? Cout_p : (Cout_p & ~7);  /* fma channels */
    for (int n = 0; n < N; ++n)
        for (int g = 0; g < groups; ++g)
            for (int oh = 0; oh < OH; ++oh)
                for (int ow = 0; ow < OW; ++ow)
                    for (int oc = 0; oc < Cout_p; ++oc) {
                        const float* wg = weight + (size_t)g * Cout_p * KH * KW * Cin_p;
                        const int fused = oc < fused_below;
                        float s = bias ? bias[g * Cout_p + oc] : 0.0f;
                        for (int kh = 0; kh < KH; ++kh) {
                            int ih = oh * stride - pad + kh;
                            if (ih < 0 || ih >= H) continue;
                            for (int kw = 0; kw < KW; ++kw) {
                                int iw = ow * stride - pad + kw;
                                if (iw < 0 || iw >= W) continue;
                                const float* ip = input + (((size_t)n * H + ih) * W + iw) * Cin + (size_t)g * Cin_p;
                                const float* wp = wg + (size_t)((kh * KW + kw) * Cin_p) * Cout_p + oc;
                                for (int ic = 0; ic < Cin_p; ++ic) {
                                    if (fused) s = fmaf(ip[ic], wp[(size_t)ic * Cout_p], s);
                                    else s += ip[ic] * wp[(size_t)ic * Cout_p];
                                }
                            }
                        }
                        if (act == 1) s = fused ? (s > 0.0f ? s : 0.0f) : (s < 0.0f ? 0.0f : s);
                        output[(((size_t)n * OH + oh) * OW + ow) * Cout + g * Cout_p + oc] = s;
                    }
}

/* winograd.cpp:31-101,167-231 — F(2,3) with Lavin's BT/G/AT, per-tile transforms,
 * accumulation over input channels in order, then bias and ReLU. */
void orc_winograd23(const float* input, int N, int H, int W, int Cin, const float* weight,
                    const float* bias, int Cout, float* output, int act) {
    const int OH = H, OW = W, tH = (OH + 1) / 2, tW = (OW + 1) / 2;
    float* gh = (float*)malloc((size_t)16 * Cin * Cout * sizeof(float));
    for (int d = 0; d < Cin; ++d)
        for (int c = 0; c < Cout; ++c) {
            float g[9], T[4][3];
            for (int k = 0; k < 9; ++k) g[k] = weight[((size_t)k * Cin + d) * Cout + c];
            for (int y = 0; y < 3; ++y) {
                float a = g[y], b = g[3 + y], cc = g[6 + y];
                T[0][y] = a; T[1][y] = 0.5f * (a + b + cc); T[2][y] = 0.5f * (a - b + cc); T[3][y] = cc;
            }
            for (int i = 0; i < 4; ++i) {
                float t0 = T[i][0], t1 = T[i][1], t2 = T[i][2];
                gh[((size_t)(i * 4 + 0) * Cin + d) * Cout + c] = t0;
                gh[((size_t)(i * 4 + 1) * Cin + d) * Cout + c] = 0.5f * (t0 + t1 + t2);
                gh[((size_t)(i * 4 + 2) * Cin + d) * Cout + c] = 0.5f * (t0 - t1 + t2);
                gh[((size_t)(i * 4 + 3) * Cin + d) * Cout + c] = t2;
            }
        }
    float* mh = (float*)malloc((size_t)16 * Cout * sizeof(float));
    for (int n = 0; n < N; ++n)
        for (int ty = 0; ty < tH; ++ty)
            for (int tx = 0; tx < tW; ++tx) {
                memset(mh, 0, (size_t)16 * Cout * sizeof(float));
                for (int d = 0; d < Cin; ++d) {
                    float dblk[16], U[4][4], dh[16];
                    for (int k = 0; k < 4; ++k)
                        for (int l = 0; l < 4; ++l) {
                            int ih = 2 * ty + k - 1, iw = 2 * tx + l - 1;
                            dblk[k * 4 + l] = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                                ? input[(((size_t)n * H + ih) * W + iw) * Cin + d] : 0.0f;
                        }
                    for (int l = 0; l < 4; ++l) {
                        float c0 = dblk[l], c1 = dblk[4 + l], c2 = dblk[8 + l], c3 = dblk[12 + l];
                        U[0][l] = c0 - c2; U[1][l] = c1 + c2; U[2][l] = -c1 + c2; U[3][l] = -c1 + c3;
                    }
                    for (int i = 0; i < 4; ++i) {
                        float u0 = U[i][0], u1 = U[i][1], u2 = U[i][2], u3 = U[i][3];
                        dh[i * 4 + 0] = u0 - u2; dh[i * 4 + 1] = u1 + u2;
                        dh[i * 4 + 2] = -u1 + u2; dh[i * 4 + 3] = -u1 + u3;
                    }
                    for (int ij = 0; ij < 16; ++ij)
                        for (int c = 0; c < Cout; ++c)
                            mh[(size_t)ij * Cout + c] = fmaf(dh[ij], gh[((size_t)ij * Cin + d) * Cout + c],
                                                             mh[(size_t)ij * Cout + c]);
                }
                static const float AT[2][4] = {{1.f, 1.f, 1.f, 0.f}, {0.f, 1.f, -1.f, 1.f}};
                for (int c = 0; c < Cout; ++c)
                    for (int r = 0; r < 2; ++r)
                        for (int cc = 0; cc < 2; ++cc) {
                            int oh = 2 * ty + r, ow = 2 * tx + cc;
                            if (oh >= OH || ow >= OW) continue;
                            float s = 0.0f;
                            for (int k = 0; k < 16; ++k)
                                s = fmaf(AT[r][k / 4] * AT[cc][k % 4], mh[(size_t)k * Cout + c], s);
                            if (bias) s = s + bias[c];
                            if (act == 1) s = fmaxf_ref(s, 0.0f);
                            output[(((size_t)n * OH + oh) * OW + ow) * Cout + c] = s;
                        }
            }
    free(gh); free(mh);
}

/* winograd43.cpp:33-96 (matrices + transforms) and winograd43_avx512.cpp:92-216. */
void orc_winograd43(const float* input, int N, int H, int W, int Cin, const float* weight,
                    const float* bias, int Cout, float* output, int act) {
    static const float BT[6][6] = {
        {4.f, 0.f, -5.f, 0.f, 1.f, 0.f}, {0.f, -4.f, -4.f, 1.f, 1.f, 0.f},
        {0.f, 4.f, -4.f, -1.f, 1.f, 0.f}, {0.f, -2.f, -1.f, 2.f, 1.f, 0.f},
        {0.f, 2.f, -1.f, -2.f, 1.f, 0.f}, {0.f, 4.f, 0.f, -5.f, 0.f, 1.f}};
    static const float G[6][3] = {
        {0.25f, 0.f, 0.f}, {-1.f / 6.f, -1.f / 6.f, -1.f / 6.f}, {-1.f / 6.f, 1.f / 6.f, -1.f / 6.f},
        {1.f / 24.f, 1.f / 12.f, 1.f / 6.f}, {1.f / 24.f, -1.f / 12.f, 1.f / 6.f}, {0.f, 0.f, 1.f}};
    static const float AT[4][6] = {
        {1.f, 1.f, 1.f, 1.f, 1.f, 0.f}, {0.f, 1.f, -1.f, 2.f, -2.f, 0.f},
        {0.f, 1.f, 1.f, 4.f, 4.f, 0.f}, {0.f, 1.f, -1.f, 8.f, -8.f, 1.f}};
    const int OH = H, OW = W, tH = (OH + 3) / 4, tW = (OW + 3) / 4;
    float* gh = (float*)malloc((size_t)36 * Cin * Cout * sizeof(float));
    for (int d = 0; d < Cin; ++d)
        for (int c = 0; c < Cout; ++c) {
            float g[9], tmp[18];
            for (int k = 0; k < 9; ++k) g[k] = weight[((size_t)k * Cin + d) * Cout + c];
            for (int i = 0; i < 6; ++i)
                for (int b = 0; b < 3; ++b) {
                    float s = 0.f;
                    for (int a = 0; a < 3; ++a) s += G[i][a] * g[a * 3 + b];
                    tmp[i * 3 + b] = s;
                }
            for (int i = 0; i < 6; ++i)
                for (int j = 0; j < 6; ++j) {
                    float s = 0.f;
                    for (int b = 0; b < 3; ++b) s += tmp[i * 3 + b] * G[j][b];
                    gh[((size_t)(i * 6 + j) * Cin + d) * Cout + c] = s;
                }
        }
    float* mh = (float*)malloc((size_t)36 * Cout * sizeof(float));
    for (int n = 0; n < N; ++n)
        for (int ty = 0; ty < tH; ++ty)
            for (int tx = 0; tx < tW; ++tx) {
                memset(mh, 0, (size_t)36 * Cout * sizeof(float));
                for (int d = 0; d < Cin; ++d) {
                    float dblk[36], tmp[36], dh[36];
                    for (int k = 0; k < 6; ++k)
                        for (int l = 0; l < 6; ++l) {
                            int ih = 4 * ty + k - 1, iw = 4 * tx + l - 1;
                            dblk[k * 6 + l] = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                                ? input[(((size_t)n * H + ih) * W + iw) * Cin + d] : 0.0f;
                        }
                    for (int i = 0; i < 6; ++i)
                        for (int b = 0; b < 6; ++b) {
                            float s = 0.f;
                            for (int a = 0; a < 6; ++a) s += BT[i][a] * dblk[a * 6 + b];
                            tmp[i * 6 + b] = s;
                        }
                    for (int i = 0; i < 6; ++i)
                        for (int j = 0; j < 6; ++j) {
                            float s = 0.f;
                            for (int b = 0; b < 6; ++b) s += tmp[i * 6 + b] * BT[j][b];
                            dh[i * 6 + j] = s;
                        }
                    for (int ij = 0; ij < 36; ++ij)
                        for (int c = 0; c < Cout; ++c)
                            mh[(size_t)ij * Cout + c] = fmaf(dh[ij], gh[((size_t)ij * Cin + d) * Cout + c],
                                                             mh[(size_t)ij * Cout + c]);
                }
                for (int c = 0; c < Cout; ++c)
                    for (int p = 0; p < 16; ++p) {
                        int a = p / 4, b = p % 4, oh = 4 * ty + a, ow = 4 * tx + b;
                        if (oh >= OH || ow >= OW) continue;
                        float s = 0.0f;
                        for (int k = 0; k < 36; ++k)
                            s = fmaf(AT[a][k / 6] * AT[b][k % 6], mh[(size_t)k * Cout + c], s);
                        if (bias) s = s + bias[c];
                        if (act == 1) s = fmaxf_ref(s, 0.0f);
                        output[(((size_t)n * OH + oh) * OW + ow) * Cout + c] = s;
                    }
            }
    free(gh); free(mh);
}

/* layers.cpp:106-195 routing decisions */
int orc_conv2d_route(int N, int H, int W, int Cin, int KH, int KW, int Cout,
                     int stride, int pad, int groups) {
    (void)N;
    if (groups > 1) {
        if (groups == Cin && groups == Cout) return 1;
        int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
        if (OH <= 0 || OW <= 0) return 0;
        if (Cin / groups <= 64 && Cout / groups <= 128) return 2;
        return 3;
    }
    if (KH == 1 && KW == 1) return 4;
    if (KH == 3 && KW == 3 && stride == 1 && pad == 1 && H >= 3 && W >= 3 && Cin >= 4 && Cout >= 4)
        return (H >= 112 && W >= 112 && Cin >= 64 && Cout >= 64) ? 5 : 6;
    int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (OH <= 0 || OW <= 0) return 0;
    return 7;
}

/* ================================================================== layers */

/* layers.cpp:19-36 (acfun_fc = GEMM + bias; acfun_fc_relu = GEMM, then bias + ReLU) */
void orc_fc(const float* input, int N, int Cin, const float* weight, const float* bias,
            int Cout, float* output, int act) {
    orc_gemm_f32(N, Cout, Cin, input, weight, output, bias, act);
}

/* layers.cpp:10-17 */
void orc_relu(float* d, size_t n) {
    for (size_t i = 0; i < n; ++i) if (d[i] < 0.0f) d[i] = 0.0f;
}
void orc_relu6(float* d, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float v = d[i];
        if (v < 0.0f) v = 0.0f; else if (v > 6.0f) v = 6.0f;
        d[i] = v;
    }
}

/* layers.cpp:221-246 (scalar) == maxpool_avx512.cpp:15-66: -1e30 sentinel, out-of-bounds
 * window cells skipped, optional post-ReLU. */
void orc_maxpool(const float* in, int N, int H, int W, int C, int pool, int stride, int pad,
                 float* out, int post_relu) {
    int OH = (H + 2 * pad - pool) / stride + 1, OW = (W + 2 * pad - pool) / stride + 1;
    if (OH <= 0 || OW <= 0) return;
    for (int n = 0; n < N; ++n)
        for (int oh = 0; oh < OH; ++oh)
            for (int ow = 0; ow < OW; ++ow)
                for (int c = 0; c < C; ++c) {
                    float mx = -1e30f;
                    for (int ph = 0; ph < pool; ++ph) {
                        int ih = oh * stride - pad + ph;
                        if (ih < 0 || ih >= H) continue;
                        for (int pw = 0; pw < pool; ++pw) {
                            int iw = ow * stride - pad + pw;
                            if (iw < 0 || iw >= W) continue;
                            float v = in[(((size_t)n * H + ih) * W + iw) * C + c];
                            if (v > mx) mx = v;
                        }
                    }
                    if (post_relu && mx < 0.0f) mx = 0.0f;
                    out[(((size_t)n * OH + oh) * OW + ow) * C + c] = mx;
                }
}

/* layers.cpp:272-283: max, expf(x - max), sequential sum, multiply by 1/sum. */
void orc_softmax(const float* in, int rows, int cols, float* out) {
    for (int r = 0; r < rows; ++r) {
        const float* ri = in + (size_t)r * cols;
        float* ro = out + (size_t)r * cols;
        float mx = ri[0];
        for (int c = 1; c < cols; ++c) if (ri[c] > mx) mx = ri[c];
        float sum = 0.0f;
        for (int c = 0; c < cols; ++c) { float e = expf(ri[c] - mx); ro[c] = e; sum += e; }
        float inv = 1.0f / sum;
        for (int c = 0; c < cols; ++c) ro[c] *= inv;
    }
}

/* layers.cpp:285-296 */
void orc_batchnorm(float* d, int size, int channels, const float* mean, const float* var,
                   const float* gamma, const float* beta, float eps) {
    int spatial = size / channels;
    for (int c = 0; c < channels; ++c) {
        float scale = gamma ? gamma[c] : 1.0f;
        float shift = beta ? beta[c] : 0.0f;
        float inv = scale / sqrtf(var[c] + eps);
        for (int s = 0; s < spatial; ++s) {
            size_t i = (size_t)s * channels + c;
            float v = d[i] - mean[c];
            v = v * inv;
            d[i] = v + shift;
        }
    }
}

/* model.cpp:69-95: scale = gamma/sqrtf(var+1e-5f), shift = beta - mean*scale, group-aware
 * weight indexing, b' = b*scale + shift. */
void orc_fold_bn(float* w, float* b, size_t wn, int Cout, int groups, const float* mean,
                 const float* var, const float* gamma, const float* beta) {
    int Cout_per = (groups > 1) ? Cout / groups : Cout;
    size_t per_in = wn / (size_t)Cout;
    for (int c = 0; c < Cout; ++c) {
        float scale = gamma[c] / sqrtf(var[c] + 1e-5f);
        float ms = mean[c] * scale;
        float shift = beta[c] - ms;
        int gc = (groups > 1) ? c / Cout_per : 0;
        int oc = (groups > 1) ? c % Cout_per : c;
        for (size_t t = 0; t < per_in; ++t) {
            size_t off = (size_t)gc * (size_t)Cout_per * per_in + t * (size_t)Cout_per + oc;
            w[off] *= scale;
        }
        float bs = b[c] * scale;
        b[c] = bs + shift;
    }
}
