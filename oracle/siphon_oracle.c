/* siphon oracle: CPU restatement of the reference's quantized matrix path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the CUDA library is
 * compared against; nothing in siphon_b200/ links, loads or calls it. It is
 * loaded by tests/, by __graft_entry__.smoke() and by bench.py's CPU
 * baseline leg, and nowhere else.
 *
 * What it restates (all paths relative to the reference project root):
 *   - f16 <-> f32 conversion ............ src/kernels.c:98-176
 *   - Q8_K activation quantizer ......... src/kernels.c:527-533, 561-595
 *   - Q8_0 activation quantizer, the
 *     AVX2 form x86 hosts dispatch to ... src/kernels_avx2.c:594-645
 *     and the scalar form ............... src/kernels.c:542-558
 *   - scalar dot products ............... src/kernels.c:189-523
 *   - row dequantisation ................ src/kernels.c:599-817
 *   - block geometry / dot pairing ...... src/kernels.c:904-919, 946-960
 *   - activation steps between products:
 *     exp polynomial, silu .............. src/kernels.c:821-853
 *     RMS scale ......................... src/kernels.c:892-900
 *     residual add, rms_norm_mul ........ src/engine.c:12-18, 369, 379
 *     swiglu_row ........................ src/engine.c:162-179
 *     attention softmax (row max, si_softmax) src/engine.c:124-130,
 *                                         src/kernels.c:855-890
 *     rope_apply, attn_head (scalar f16
 *     dots), the f16 cache writes ........ src/engine.c:42-75, 90-147, 344-362
 *
 * Integer partial sums are order-free, so they are written here in whatever
 * order reads best. Every floating-point operation is written one rounding
 * at a time in exactly the order the reference's scalar code performs it;
 * the file must be compiled with -ffp-contract=off (oracle/Makefile does)
 * so no multiply-add is fused.
 *
 * Parity pin: tests/test_oracle_pin.py compares every function here with
 * the reference built from its own sources (oracle/_ref), and
 * tests/test_oracle_golden.py against fixtures that reference produced
 * (tests/golden/gen_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ggml type ids as stored in GGUF (include/siphon/quant.h:103-119) */
enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
    T_Q8_K = 15,
};

/* on-disk block sizes (include/siphon/quant.h:92-100) */
enum {
    B_Q4_0 = 18, B_Q5_0 = 22, B_Q8_0 = 34, B_Q2_K = 84, B_Q3_K = 110,
    B_Q4_K = 144, B_Q5_K = 176, B_Q6_K = 210, B_Q8_K = 292,
};

static inline uint16_t ld16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t ld32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float ldf32(const uint8_t *p) { return bits_f32(ld32(p)); }

/* ---- half precision ------------------------------------------------------
 * kernels.c:98-122 widens exactly (NaN payloads kept, not quieted). A half
 * with a zero exponent field is man * 2^-24, which a float holds exactly. */
ORC_API float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 31) return bits_f32(sign | 0x7f800000u | (m << 13));
    if (e == 0) {
        const float mag = ldexpf((float)m, -24);
        return sign ? -mag : mag;
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* kernels.c:124-176: IEEE round-to-nearest-even narrowing; a NaN becomes
 * sign|0x7c00|0x0200|payload>>13 (payload forced non-zero). */
ORC_API uint16_t orc_f32_to_f16(float f) {
    const uint32_t u = f32_bits(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t ef = (u >> 23) & 0xffu, m = u & 0x7fffffu;
    if (ef == 0xff) {
        if (m == 0) return (uint16_t)(sign | 0x7c00u);
        uint32_t p = m >> 13;
        if (p == 0) p = 1;
        return (uint16_t)(sign | 0x7c00u | 0x0200u | p);
    }
    const int e = (int)ef - 112;               /* biased half exponent */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;              /* below half the smallest subnormal */
        const uint32_t full = m | 0x800000u;   /* implicit bit made explicit */
        const int drop = 14 - e;               /* 14..24 bits go away */
        uint32_t q = full >> drop;
        const uint32_t rest = full & ((1u << drop) - 1u), mid = 1u << (drop - 1);
        if (rest > mid || (rest == mid && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (q & 1u))) q++;   /* may carry into inf */
    return (uint16_t)(sign | q);
}

/* ---- geometry (kernels.c:904-919) and dot pairing (kernels.c:946-960) ---- */
ORC_API int orc_geometry(uint32_t t, uint32_t *blck, uint32_t *bytes) {
    static const struct { uint32_t t, n, b; } g[] = {
        {T_F32, 1, 4}, {T_F16, 1, 2}, {T_Q4_0, 32, B_Q4_0}, {T_Q5_0, 32, B_Q5_0},
        {T_Q8_0, 32, B_Q8_0}, {T_Q2_K, 256, B_Q2_K}, {T_Q3_K, 256, B_Q3_K},
        {T_Q4_K, 256, B_Q4_K}, {T_Q5_K, 256, B_Q5_K}, {T_Q6_K, 256, B_Q6_K},
        {T_Q8_K, 256, B_Q8_K},
    };
    for (unsigned i = 0; i < sizeof g / sizeof g[0]; i++) {
        if (g[i].t == t) { *blck = g[i].n; *bytes = g[i].b; return 1; }
    }
    return 0;
}

ORC_API int orc_pair_type(uint32_t wt, uint32_t *pair) {
    switch (wt) {
        case T_F32: case T_F16: *pair = wt; return 1;
        case T_Q4_0: case T_Q5_0: case T_Q8_0: *pair = T_Q8_0; return 1;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: *pair = T_Q8_K; return 1;
        default: return 0;
    }
}

/* ---- activation quantizers ------------------------------------------------ */

/* Q8_K, kernels.c:561-595. Per 256: the first element of largest magnitude
 * (strict > scan) fixes iscale = -127/max; quants are nearest_int(iscale*x)
 * capped at +127, bsums are the 16-element group sums, d = 1/iscale.
 * nearest_int (kernels.c:528-533) is the 1.5*2^23 magic add: round half to
 * even for every product that can occur here. On x86 a NaN product is the
 * NaN operand itself, so the magic add leaves its low 22 payload bits as
 * the "integer"; that is reproduced for NaN inputs. An all-zero block sets
 * d = 0 and qs = 0 and leaves bsums as they were (kernels.c:574-579). */
ORC_API void orc_quant_q8_K(const float *x, uint8_t *y, int n) {
    for (int b = 0; b < n / 256; b++, x += 256, y += B_Q8_K) {
        float peak = 0.0f, lead = 0.0f;
        for (int j = 0; j < 256; j++) {
            const float a = fabsf(x[j]);
            if (a > peak) { peak = a; lead = x[j]; }
        }
        int8_t *qs = (int8_t *)(y + 4);
        if (peak == 0.0f) {
            const float zero = 0.0f;
            memcpy(y, &zero, 4);
            memset(qs, 0, 256);
            continue;
        }
        const float iscale = -127.f / lead;
        for (int j = 0; j < 256; j++) {
            int v;
            if (isnan(x[j])) {
                v = (int)(f32_bits(x[j]) & 0x3fffffu);
            } else {
                const float p = iscale * x[j];
                v = (int)((f32_bits(p + 12582912.f) & 0x7fffffu)) - 0x400000;
            }
            qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int k = 0; k < 16; k++) s += qs[16 * g + k];
            const int16_t s16 = (int16_t)s;
            memcpy(y + 260 + 2 * g, &s16, 2);
        }
        const float d = 1.0f / iscale;
        memcpy(y, &d, 4);
    }
}

/* vmaxps semantics: first operand if it compares greater, else the second
 * (so a NaN in either slot yields the second operand). */
static inline float vmax(float a, float b) { return a > b ? a : b; }

/* int32 -> int16 -> int8 with saturation at each step, as packs_epi32 then
 * packs_epi16 do; a NaN / out-of-range cvtps_epi32 gives INT32_MIN. */
static inline int8_t sat8_from_rounded(float r) {
    int32_t i;
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) i = INT32_MIN;
    else i = (int32_t)r;
    if (i > 127) i = 127;
    if (i < -128) i = -128;
    return (int8_t)i;
}

/* Q8_0 in the AVX2 form that x86 hosts run (kernels_avx2.c:594-645): the
 * lane-wise max tree of |x|, d = max/127 stored as f16, id = 127/max,
 * quants = round-half-even(x*id) with saturating packs. */
ORC_API void orc_quant_q8_0(const float *x, uint8_t *y, int n) {
    for (int b = 0; b < n / 32; b++, x += 32, y += B_Q8_0) {
        float lane[8];
        for (int i = 0; i < 8; i++) {
            float m = fabsf(x[i]);
            m = vmax(m, fabsf(x[8 + i]));
            m = vmax(m, fabsf(x[16 + i]));
            m = vmax(m, fabsf(x[24 + i]));
            lane[i] = m;
        }
        float q4[4];
        for (int i = 0; i < 4; i++) q4[i] = vmax(lane[4 + i], lane[i]);
        const float q2a = vmax(q4[0], q4[2]), q2b = vmax(q4[1], q4[3]);
        const float top = vmax(q2a, q2b);
        const uint16_t dh = orc_f32_to_f16(top / 127.f);
        y[0] = (uint8_t)dh; y[1] = (uint8_t)(dh >> 8);
        const float id = (top != 0.0f) ? 127.f / top : 0.0f;
        for (int j = 0; j < 32; j++) y[2 + j] = (uint8_t)sat8_from_rounded(nearbyintf(x[j] * id));
    }
}

/* Q8_0 in the portable scalar form (kernels.c:542-558): id = 1/(amax/127)
 * and roundf (half away from zero). Kept to report how often the two forms
 * disagree; the CUDA quantizer follows the AVX2 form above. */
ORC_API void orc_quant_q8_0_scalar(const float *x, uint8_t *y, int n) {
    for (int b = 0; b < n / 32; b++, x += 32, y += B_Q8_0) {
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = amax > fabsf(x[j]) ? amax : fabsf(x[j]);
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = orc_f32_to_f16(d);
        y[0] = (uint8_t)dh; y[1] = (uint8_t)(dh >> 8);
        for (int j = 0; j < 32; j++) y[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
    }
}

/* F16 pair: element-wise RNE narrowing (src/backend.c:19-27) */
ORC_API void orc_convert_f16(const float *x, uint16_t *y, int n) {
    for (int i = 0; i < n; i++) y[i] = orc_f32_to_f16(x[i]);
}

/* ---- weight element decoders ----------------------------------------------
 * One function per format returning the signed integer quant of element e
 * (0..255 within a super-block, 0..31 within a classic block) and, for the
 * K formats, the scale (and min) of the sub-block e falls in. */

/* Q4_K/Q5_K 6-bit scale/min unpack (kernels.c:648-656, identical to the
 * utmp shuffle at kernels.c:377-382) */
static void k4_scales(const uint8_t *s, int sc[8], int mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 15) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
}

/* Q4_K element (kernels.c:371-376): chunk c = e/64 of 32 bytes; low nibble
 * for e%64 < 32, high nibble otherwise */
static int q4k_elem(const uint8_t *blk, int e) {
    const uint8_t byte = blk[16 + 32 * (e / 64) + (e % 32)];
    return (e % 64) < 32 ? (byte & 15) : (byte >> 4);
}

/* Q5_K element (kernels.c:436-444): Q4_K nibble + 16 * bit (e/32) of qh[e%32] */
static int q5k_elem(const uint8_t *blk, int e) {
    const uint8_t byte = blk[48 + 32 * (e / 64) + (e % 32)];
    const int nib = (e % 64) < 32 ? (byte & 15) : (byte >> 4);
    return nib + (((blk[16 + e % 32] >> (e / 32)) & 1) ? 16 : 0);
}

/* Q6_K element (kernels.c:496-506): half h, group g of 32, lane i */
static int q6k_elem(const uint8_t *blk, int e) {
    const int h = e / 128, g = (e % 128) / 32, i = e % 32;
    const uint8_t lo = blk[64 * h + i + ((g & 1) ? 32 : 0)];
    const uint8_t hi = blk[128 + 32 * h + i];
    const int nib = g < 2 ? (lo & 15) : (lo >> 4);
    return (nib | (((hi >> (2 * g)) & 3) << 4)) - 32;
}

/* Q3_K element (kernels.c:311-325): 2-bit quant, minus 4 when the hmask bit
 * (4h + g) of hmask[i] is clear */
static int q3k_elem(const uint8_t *blk, int e) {
    const int h = e / 128, g = (e % 128) / 32, i = e % 32;
    const int q = (blk[32 + 32 * h + i] >> (2 * g)) & 3;
    return q - ((blk[i] >> (4 * h + g)) & 1 ? 0 : 4);
}

/* Q3_K 6-bit scales (kernels.c:328-333): low nibble from byte j (j<8) or
 * the high nibble of byte j-8, top two bits from byte 8 + j%4 at 2*(j/4) */
static void q3k_scales(const uint8_t *blk, int sc[16]) {
    const uint8_t *s = blk + 96;
    for (int j = 0; j < 16; j++) {
        const int lo = j < 8 ? (s[j] & 15) : (s[j - 8] >> 4);
        const int hi = (s[8 + j % 4] >> (2 * (j / 4))) & 3;
        sc[j] = (lo | (hi << 4)) - 32;
    }
}

/* Q2_K element (kernels.c:268-283): half k, shift group jj, 16-lane half */
static int q2k_elem(const uint8_t *blk, int e) {
    const int k = e / 128, r = e % 128, jj = r / 32, i = r % 32;
    return (blk[16 + 32 * k + i] >> (2 * jj)) & 3;
}

/* ---- dot products (scalar reference semantics) ------------------------------ */

/* Shared tail of the K formats with eight lane accumulators
 * (kernels.c:343-345, 403-408, 471-476, 518-521): per super-block
 * sums[l] += d * aux[l]; after the row, sumf += sums[l] for l = 0..7. */
typedef struct { float sums[8]; float sumf; } lanes8;

static void lanes8_add(lanes8 *st, float d, const int32_t aux[8]) {
    for (int l = 0; l < 8; l++) st->sums[l] = st->sums[l] + d * (float)aux[l];
}
static float lanes8_finish(lanes8 *st) {
    float s = st->sumf;
    for (int l = 0; l < 8; l++) s = s + st->sums[l];
    return s;
}

/* kernels.c:349-410 */
ORC_API float orc_dot_q4_K(int n, const uint8_t *x, const uint8_t *y) {
    lanes8 st = {{0}, 0.0f};
    for (int i = 0; i < n / 256; i++, x += B_Q4_K, y += B_Q8_K) {
        int sc[8], mn[8];
        k4_scales(x + 4, sc, mn);
        const int8_t *a = (const int8_t *)(y + 4);
        int32_t aux[8] = {0};
        for (int e = 0; e < 256; e++) aux[e % 8] += sc[e / 32] * (q4k_elem(x, e) * a[e]);
        int mins = 0;
        for (int g = 0; g < 16; g++) {
            int16_t bs; memcpy(&bs, y + 260 + 2 * g, 2);
            mins += bs * mn[g / 2];
        }
        const float yd = ldf32(y);
        lanes8_add(&st, orc_f16_to_f32(ld16(x)) * yd, aux);
        st.sumf = st.sumf - (orc_f16_to_f32(ld16(x + 2)) * yd) * (float)mins;
    }
    return lanes8_finish(&st);
}

/* kernels.c:412-478 */
ORC_API float orc_dot_q5_K(int n, const uint8_t *x, const uint8_t *y) {
    lanes8 st = {{0}, 0.0f};
    for (int i = 0; i < n / 256; i++, x += B_Q5_K, y += B_Q8_K) {
        int sc[8], mn[8];
        k4_scales(x + 4, sc, mn);
        const int8_t *a = (const int8_t *)(y + 4);
        int32_t aux[8] = {0};
        for (int e = 0; e < 256; e++) aux[e % 8] += sc[e / 32] * (q5k_elem(x, e) * a[e]);
        int mins = 0;
        for (int g = 0; g < 16; g++) {
            int16_t bs; memcpy(&bs, y + 260 + 2 * g, 2);
            mins += bs * mn[g / 2];
        }
        const float yd = ldf32(y);
        lanes8_add(&st, orc_f16_to_f32(ld16(x)) * yd, aux);
        st.sumf = st.sumf - (orc_f16_to_f32(ld16(x + 2)) * yd) * (float)mins;
    }
    return lanes8_finish(&st);
}

/* kernels.c:480-523 */
ORC_API float orc_dot_q6_K(int n, const uint8_t *x, const uint8_t *y) {
    lanes8 st = {{0}, 0.0f};
    for (int i = 0; i < n / 256; i++, x += B_Q6_K, y += B_Q8_K) {
        const int8_t *sc = (const int8_t *)(x + 192);
        const int8_t *a = (const int8_t *)(y + 4);
        int32_t aux[8] = {0};
        for (int e = 0; e < 256; e++) aux[e % 8] += sc[e / 16] * (q6k_elem(x, e) * a[e]);
        lanes8_add(&st, orc_f16_to_f32(ld16(x + 208)) * ldf32(y), aux);
    }
    return lanes8_finish(&st);
}

/* kernels.c:289-347 */
ORC_API float orc_dot_q3_K(int n, const uint8_t *x, const uint8_t *y) {
    lanes8 st = {{0}, 0.0f};
    for (int i = 0; i < n / 256; i++, x += B_Q3_K, y += B_Q8_K) {
        int sc[16];
        q3k_scales(x, sc);
        const int8_t *a = (const int8_t *)(y + 4);
        int32_t aux[8] = {0};
        for (int e = 0; e < 256; e++) aux[e % 8] += sc[e / 16] * (q3k_elem(x, e) * a[e]);
        lanes8_add(&st, orc_f16_to_f32(ld16(x + 108)) * ldf32(y), aux);
    }
    return lanes8_finish(&st);
}

/* kernels.c:249-287: one integer sum per super-block, then
 * sumf += dall*isum - dmin*summs */
ORC_API float orc_dot_q2_K(int n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0.0f;
    for (int i = 0; i < n / 256; i++, x += B_Q2_K, y += B_Q8_K) {
        const int8_t *a = (const int8_t *)(y + 4);
        int isum = 0, summs = 0;
        for (int e = 0; e < 256; e++) isum += (x[e / 16] & 15) * (q2k_elem(x, e) * a[e]);
        for (int g = 0; g < 16; g++) {
            int16_t bs; memcpy(&bs, y + 260 + 2 * g, 2);
            summs += bs * (x[g] >> 4);
        }
        const float yd = ldf32(y);
        const float dall = yd * orc_f16_to_f32(ld16(x + 80));
        const float dmin = yd * orc_f16_to_f32(ld16(x + 82));
        sumf = sumf + (dall * (float)isum - dmin * (float)summs);
    }
    return sumf;
}

/* kernels.c:197-213: sumf += sumi * dx * dy, left to right */
ORC_API float orc_dot_q4_0(int n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0.0f;
    for (int b = 0; b < n / 32; b++, x += B_Q4_0, y += B_Q8_0) {
        const int8_t *a = (const int8_t *)(y + 2);
        int s = 0;
        for (int j = 0; j < 16; j++) s += ((x[2 + j] & 15) - 8) * a[j] + ((x[2 + j] >> 4) - 8) * a[j + 16];
        sumf = sumf + ((float)s * orc_f16_to_f32(ld16(x))) * orc_f16_to_f32(ld16(y));
    }
    return sumf;
}

/* kernels.c:215-233: bit j of qh tops element j, bit j+16 element j+16 */
ORC_API float orc_dot_q5_0(int n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0.0f;
    for (int b = 0; b < n / 32; b++, x += B_Q5_0, y += B_Q8_0) {
        const int8_t *a = (const int8_t *)(y + 2);
        const uint32_t qh = ld32(x + 2);
        int s = 0;
        for (int j = 0; j < 16; j++) {
            const int v0 = ((x[6 + j] & 15) | (int)(((qh >> j) & 1) << 4)) - 16;
            const int v1 = ((x[6 + j] >> 4) | (int)(((qh >> (j + 16)) & 1) << 4)) - 16;
            s += v0 * a[j] + v1 * a[j + 16];
        }
        sumf = sumf + ((float)s * orc_f16_to_f32(ld16(x))) * orc_f16_to_f32(ld16(y));
    }
    return sumf;
}

/* kernels.c:235-247: sumf += sumi * (dx * dy) */
ORC_API float orc_dot_q8_0(int n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0.0f;
    for (int b = 0; b < n / 32; b++, x += B_Q8_0, y += B_Q8_0) {
        const int8_t *w = (const int8_t *)(x + 2), *a = (const int8_t *)(y + 2);
        int s = 0;
        for (int j = 0; j < 32; j++) s += w[j] * a[j];
        sumf = sumf + (float)s * (orc_f16_to_f32(ld16(x)) * orc_f16_to_f32(ld16(y)));
    }
    return sumf;
}

/* kernels.c:189-195: float products summed into a double, left to right */
ORC_API float orc_dot_f16(int n, const uint8_t *x, const uint8_t *y) {
    double acc = 0.0;
    for (int i = 0; i < n; i++) {
        acc += (double)(orc_f16_to_f32(ld16(x + 2 * i)) * orc_f16_to_f32(ld16(y + 2 * i)));
    }
    return (float)acc;
}

/* kernels.c:180-187 (F32 rows are not on the quantized path; kept so the
 * gemv below accepts every type the reference's cpu_gemv does) */
ORC_API float orc_dot_f32(int n, const uint8_t *x, const uint8_t *y) {
    double acc = 0.0;
    for (int i = 0; i < n; i++) acc += (double)(ldf32(x + 4 * i) * ldf32(y + 4 * i));
    return (float)acc;
}

typedef float (*dot_fn)(int, const uint8_t *, const uint8_t *);

static dot_fn dot_for(uint32_t wt) {
    switch (wt) {
        case T_F32: return orc_dot_f32;
        case T_F16: return orc_dot_f16;
        case T_Q4_0: return orc_dot_q4_0;
        case T_Q5_0: return orc_dot_q5_0;
        case T_Q8_0: return orc_dot_q8_0;
        case T_Q2_K: return orc_dot_q2_K;
        case T_Q3_K: return orc_dot_q3_K;
        case T_Q4_K: return orc_dot_q4_K;
        case T_Q5_K: return orc_dot_q5_K;
        case T_Q6_K: return orc_dot_q6_K;
        default: return 0;
    }
}

/* One dot of a weight row against an already converted activation. */
ORC_API int orc_vec_dot(uint32_t wt, int n, const void *x, const void *y, float *s) {
    dot_fn f = dot_for(wt);
    if (!f) return -4;
    *s = f(n, (const uint8_t *)x, (const uint8_t *)y);
    return 0;
}

/* Convert an f32 activation row into wt's pair format (src/backend.c:17-47). */
ORC_API int orc_quantize_pair(uint32_t wt, const float *x, void *out, int n) {
    uint32_t pair;
    if (!orc_pair_type(wt, &pair)) return -4;
    switch (pair) {
        case T_F32: memcpy(out, x, (size_t)n * 4); return 0;
        case T_F16: orc_convert_f16(x, (uint16_t *)out, n); return 0;
        case T_Q8_0: orc_quant_q8_0(x, (uint8_t *)out, n); return 0;
        default: orc_quant_q8_K(x, (uint8_t *)out, n); return 0;
    }
}

/* Rows [r0, r1) of y = W xq, W row-major [n_out, n_in] of wt blocks,
 * xq already in the pair format (src/backend.c:61-71). */
ORC_API int orc_gemv_rows(uint32_t wt, const void *w, int64_t row_bytes, int n_in,
                          int64_t r0, int64_t r1, const void *xq, float *y) {
    dot_fn f = dot_for(wt);
    if (!f) return -4;
    const uint8_t *base = (const uint8_t *)w;
    for (int64_t r = r0; r < r1; r++) y[r] = f(n_in, base + r * row_bytes, (const uint8_t *)xq);
    return 0;
}

/* ---- dequantisation (kernels.c:599-817), the row_to_f32 leg ------------------ */

ORC_API int orc_dequant_row(uint32_t t, const void *xv, float *y, int n) {
    const uint8_t *x = (const uint8_t *)xv;
    switch (t) {
        case T_F32: memcpy(y, x, (size_t)n * 4); return 0;
        case T_F16:
            for (int i = 0; i < n; i++) y[i] = orc_f16_to_f32(ld16(x + 2 * i));
            return 0;
        case T_Q4_0:
            for (int b = 0; b < n / 32; b++, x += B_Q4_0) {
                const float d = orc_f16_to_f32(ld16(x));
                for (int j = 0; j < 16; j++) {
                    y[32 * b + j] = (float)((x[2 + j] & 15) - 8) * d;
                    y[32 * b + j + 16] = (float)((x[2 + j] >> 4) - 8) * d;
                }
            }
            return 0;
        case T_Q5_0:
            for (int b = 0; b < n / 32; b++, x += B_Q5_0) {
                const float d = orc_f16_to_f32(ld16(x));
                const uint32_t qh = ld32(x + 2);
                for (int j = 0; j < 16; j++) {
                    y[32 * b + j] = (float)(((x[6 + j] & 15) | (int)(((qh >> j) & 1) << 4)) - 16) * d;
                    y[32 * b + j + 16] = (float)(((x[6 + j] >> 4) | (int)(((qh >> (j + 16)) & 1) << 4)) - 16) * d;
                }
            }
            return 0;
        case T_Q8_0:
            for (int b = 0; b < n / 32; b++, x += B_Q8_0) {
                const float d = orc_f16_to_f32(ld16(x));
                for (int j = 0; j < 32; j++) y[32 * b + j] = (float)(int8_t)x[2 + j] * d;
            }
            return 0;
        case T_Q2_K:
            /* kernels.c:658-682: dl * q - ml per 16 elements */
            for (int b = 0; b < n / 256; b++, x += B_Q2_K) {
                const float d = orc_f16_to_f32(ld16(x + 80)), mn = orc_f16_to_f32(ld16(x + 82));
                for (int e = 0; e < 256; e++) {
                    const uint8_t s = x[e / 16];
                    const float dl = d * (float)(s & 15), ml = mn * (float)(s >> 4);
                    y[256 * b + e] = dl * (float)q2k_elem(x, e) - ml;
                }
            }
            return 0;
        case T_Q3_K:
            for (int b = 0; b < n / 256; b++, x += B_Q3_K) {
                int sc[16];
                q3k_scales(x, sc);
                const float d = orc_f16_to_f32(ld16(x + 108));
                for (int e = 0; e < 256; e++) y[256 * b + e] = (d * (float)sc[e / 16]) * (float)q3k_elem(x, e);
            }
            return 0;
        case T_Q4_K:
        case T_Q5_K:
            /* kernels.c:726-774: d*sc * q - dmin*m */
            for (int b = 0; b < n / 256; b++) {
                int sc[8], mn[8];
                k4_scales(x + 4, sc, mn);
                const float d = orc_f16_to_f32(ld16(x)), dm = orc_f16_to_f32(ld16(x + 2));
                for (int e = 0; e < 256; e++) {
                    const int q = t == T_Q4_K ? q4k_elem(x, e) : q5k_elem(x, e);
                    y[256 * b + e] = (d * (float)sc[e / 32]) * (float)q - dm * (float)mn[e / 32];
                }
                x += t == T_Q4_K ? B_Q4_K : B_Q5_K;
            }
            return 0;
        case T_Q6_K:
            /* kernels.c:776-801: y = d * sc * q (left to right) */
            for (int b = 0; b < n / 256; b++, x += B_Q6_K) {
                const float d = orc_f16_to_f32(ld16(x + 208));
                const int8_t *sc = (const int8_t *)(x + 192);
                for (int e = 0; e < 256; e++) y[256 * b + e] = (d * (float)sc[e / 16]) * (float)q6k_elem(x, e);
            }
            return 0;
        default:
            return -4;
    }
}

/* ---- activation steps between the products ----------------------------------
 * The residual add, RMS norm and SwiGLU the reference's forward pass runs on
 * the host between two gemv calls (src/engine.c:12-18, 162-179, 369, 379). */

/* exp polynomial, src/kernels.c:821-849: round x / ln2 to n with the 1.5 * 2^23
 * shifter, reduce b = x - n ln2 (ln2 split in two), degree-5 polynomial p(b),
 * result 2^n (1 + p); two-factor scaling past |n| = 126, saturation past 192. */
ORC_API float orc_expf(float x) {
    const float shift = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, shift);
    const float n = z - shift;
    const float b = fmaf(-n, 0x1.7f7d1cp-20f, fmaf(-n, 0x1.62e4p-1f, x));
    const uint32_t e = f32_bits(z) << 23;
    const float two_n = bits_f32(e + 0x3f800000u);
    const float b2 = b * b;
    const float p45 = fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f);
    const float p23 = fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f);
    const float p1 = 0x1.ffffecp-1f * b;
    const float p = fmaf(fmaf(p45, b2, p23), b2, p1);
    if (!(fabsf(n) > 126.0f)) return fmaf(p, two_n, two_n);
    const uint32_t g = n <= 0.0f ? 0x82000000u : 0u;
    const float s1 = bits_f32(g + 0x7f000000u);
    if (fabsf(n) > 192.0f) return s1 * s1;
    const float s2 = bits_f32(e - g);
    return fmaf(s2, p, s2) * s1;
}

/* src/kernels.c:851-853 */
ORC_API float orc_silu(float x) { return x / (1.0f + orc_expf(0.0f - x)); }

/* src/kernels.c:892-900: f32 squares summed in double in index order */
ORC_API float orc_rms_scale(const float *x, int n, float eps) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / n);
    return 1.0f / sqrtf(mean + eps);
}

/* residual add (src/engine.c:369, 379; res may be NULL) into h, then
 * rms_norm_mul (src/engine.c:12-18) into y */
ORC_API void orc_rms_norm(const float *x, const float *res, float *h, const float *w, int n, float eps, float *y) {
    for (int i = 0; i < n; i++) h[i] = res ? x[i] + res[i] : x[i];
    const float scale = orc_rms_scale(h, n, eps);
    for (int i = 0; i < n; i++) y[i] = h[i] * scale * w[i];
}

/* swiglu_row (src/engine.c:162-179): 8-wide groups through the polynomial,
 * the n % 8 tail through libm's expf */
ORC_API void orc_swiglu(const float *x, const float *g, int n, float *y) {
    const int body = n - n % 8;
    int i = 0;
    for (; i < body; i++) y[i] = orc_silu(x[i]) * g[i];
    for (; i < n; i++) y[i] = x[i] / (1.0f + expf(0.0f - x[i])) * g[i];
}

/* the attention's softmax: the row maximum (src/engine.c:124-128), then
 * si_softmax (src/kernels.c:855-890): 8-wide groups through the polynomial,
 * each group's lanes summed as the AVX2 horizontal add orders them, into a
 * double; the n % 8 tail through libm's expf; y *= (float)(1 / sum) */
ORC_API void orc_softmax(const float *x, float *y, int n) {
    float max = -INFINITY;
    for (int j = 0; j < n; j++)
        if (x[j] > max) max = x[j];
    double sum = 0;
    int i = 0;
    for (; i + 7 < n; i += 8) {
        float v[8];
        for (int k = 0; k < 8; k++) v[k] = orc_expf(x[i + k] - max);
        for (int k = 0; k < 8; k++) y[i + k] = v[k];
        const float s0 = v[4] + v[0], s1 = v[5] + v[1], s2 = v[6] + v[2], s3 = v[7] + v[3];
        const float t0 = s0 + s2, t1 = s1 + s3;
        sum += (double)(t0 + t1);
    }
    for (; i < n; ++i) {
        const float val = expf(x[i] - max);
        sum += (double)val;
        y[i] = val;
    }
    const float scale = (float)(1.0 / sum);
    for (i = 0; i < n; ++i) y[i] *= scale;
}

/* The device softmax's restatement of libm's expf (the table-driven
 * algorithm of this image's glibc, FMA build), for checking that algorithm
 * against the host's expf on the CPU. Not used by the other functions here,
 * which call libm itself as the reference does. */
static const uint64_t orc_exp2tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};
ORC_API float orc_expf_libm_restated(float x) {
    const uint32_t ux = f32_bits(x), abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= (f32_bits(88.0f) >> 20)) {
        if (ux == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8u) return x + x;
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double invln2n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
    const double xd = (double)x, z = invln2n * xd;
    double kd = z + shift;
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= shift;
    const double r = fma(invln2n, xd, -kd);
    uint64_t t = orc_exp2tab[ki % 32] + (ki << 47);
    double sv;
    memcpy(&sv, &t, 8);
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                 c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double p = fma(c0, r, c1), r2 = r * r;
    double y = fma(c2, r, 1.0);
    y = fma(p, r2, y);
    return (float)(y * sv);
}

/* count of inputs in [lo_bits, hi_bits] (stride) where the restatement and
 * libm's expf differ */
ORC_API long orc_expf_restated_mismatches(uint32_t lo_bits, uint32_t hi_bits, uint32_t stride) {
    long bad = 0;
    for (uint64_t u = lo_bits; u <= hi_bits; u += stride) {
        const float x = bits_f32((uint32_t)u);
        if (f32_bits(expf(x)) != f32_bits(orc_expf_libm_restated(x))) bad++;
    }
    return bad;
}

/* rope_table (src/engine.c:26-40) for positions 0..n_pos-1 with the engine's
 * theta_scale = powf(base, -2.0f / n_rot) (src/engine.c:196), no frequency
 * factors: cs / sn [n_pos][n_rot / 2] */
ORC_API void orc_rope_table(float base, int n_rot, int n_pos, float *cs, float *sn) {
    const float theta_scale = powf(base, -2.0f / (float)n_rot);
    const int np = n_rot / 2;
    for (int p = 0; p < n_pos; p++) {
        float theta = (float)p;
        for (int j = 0; j < np; j++) {
            cs[(size_t)p * np + j] = cosf(theta);
            sn[(size_t)p * np + j] = sinf(theta);
            theta *= theta_scale;
        }
    }
}

/* rope_apply (src/engine.c:42-75) on n_heads heads in place */
ORC_API void orc_rope(float *x, int n_heads, int hd, int n_rot, const float *cs, const float *sn, int neox) {
    const int np = n_rot / 2;
    for (int hh = 0; hh < n_heads; hh++) {
        float *v = x + (size_t)hh * hd;
        for (int j = 0; j < np; j++) {
            if (!neox) {
                const float x0 = v[2 * j], x1 = v[2 * j + 1];
                v[2 * j] = fmaf(x0, cs[j], -(x1 * sn[j]));
                v[2 * j + 1] = fmaf(x0, sn[j], x1 * cs[j]);
            } else {
                const int half = hd / 2;
                const float x0 = v[j], x1 = v[j + half];
                v[j] = x0 * cs[j] - x1 * sn[j];
                v[j + half] = x0 * sn[j] + x1 * cs[j];
            }
        }
    }
}

static float dot_f16_scalar(int n, const uint16_t *x, size_t sx, const uint16_t *y) {
    double s = 0.0;
    for (int i = 0; i < n; i++) s += (double)(orc_f16_to_f32(x[(size_t)i * sx]) * orc_f16_to_f32(y[i]));
    return (float)s;
}

/* attn_head (src/engine.c:90-147) for every query head, with the scalar
 * si_dot_f16 (src/kernels.c:189-195) the reference runs under SI_SCALAR;
 * caches in the engine's layout (src/engine.c:344-362) */
ORC_API void orc_attention(const float *q, const uint16_t *kc, const uint16_t *vc, int n_head, int n_head_kv, int hd,
                           int n_ctx, int pos, float ks, float *out) {
    const int n_score = pos + 1, gqa = n_head / n_head_kv;
    float *sc = malloc(sizeof(float) * (size_t)n_score), *pr = malloc(sizeof(float) * (size_t)n_score);
    uint16_t *pr16 = malloc(2 * (size_t)n_score), *q16 = malloc(2 * (size_t)hd);
    for (int h = 0; h < n_head; h++) {
        const int hk = h / gqa;
        const uint16_t *kh = kc + (size_t)hk * n_ctx * hd, *vh = vc + (size_t)hk * hd * n_ctx;
        for (int d = 0; d < hd; d++) q16[d] = orc_f32_to_f16(q[(size_t)h * hd + d]);
        for (int j = 0; j < n_score; j++) sc[j] = dot_f16_scalar(hd, kh + (size_t)j * hd, 1, q16);
        for (int j = 0; j < n_score; j++) sc[j] = sc[j] * ks;
        orc_softmax(sc, pr, n_score);
        for (int j = 0; j < n_score; j++) pr16[j] = orc_f32_to_f16(pr[j]);
        for (int c = 0; c < hd; c++) out[(size_t)h * hd + c] = dot_f16_scalar(n_score, vh + (size_t)c * n_ctx, 1, pr16);
    }
    free(sc); free(pr); free(pr16); free(q16);
}
