/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the ASTC-KV decode path.
 *
 * This file is the checker, never the product: only tests/, the smoke entry
 * point and bench.py's CPU-baseline leg load it. The shipped decode path is the
 * CUDA library under astc-kv_b200/csrc.
 *
 * What it restates. The reference decodes blocks with Arm astcenc 5.7.0
 * through astc_kv/bridge.cpp:27-35 (`akv_decode`, F32 RGBA output, LDR
 * profile, swizzle RGBA) called from astc_kv/codec.py:45-59. astcenc itself is
 * not vendored in the reference tree (fetched by
 * scripts/download_dependencies.py:379-382, tarball SHA256 7c1b28ec...), so
 * this is a plain-C restatement of the published algorithm the library
 * implements: the Khronos Data Format Specification, ASTC chapter, for 2D LDR
 * blocks (block-mode table, BISE trit/quint integer coding, colour and weight
 * unquantisation, partition hash, LDR endpoint modes 0/1/4/5/6/8/9/10/12/13,
 * weight-grid infill, dual plane, void-extent blocks and the error colour).
 *
 * Outputs per texel and channel: the 16-bit interpolation result C (UNORM16),
 * its decode_unorm8 view (C >> 8) and its decode_float16 view (C == 65535 ->
 * 1.0, else C/65536 rounded toward zero to fp16). The fp16 view is what
 * astcenc's F32 LDR output carries; it is pinned against the reference's
 * golden `*_decoded.f32` files by tests/test_oracle_golden.py.
 *
 * HDR endpoint modes and HDR void-extent blocks return the error colour
 * (the LDR-profile rule).
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <pthread.h>

#define AO_OK 0
#define AO_ERROR_BLOCK 1
#define AO_VOID_EXTENT 2

/* ---------------------------------------------------------------- bits ---- */

/* Read `count` (<= 32) bits starting at bit `start` of a 128-bit little-endian
 * block; bits past 127 read as zero. */
static uint32_t rd(const uint8_t *b, int start, int count)
{
    uint32_t v = 0;
    for (int i = 0; i < count; i++) {
        int p = start + i;
        if (p >= 0 && p < 128 && ((b[p >> 3] >> (p & 7)) & 1))
            v |= 1u << i;
    }
    return v;
}

static void reverse128(const uint8_t *in, uint8_t *out)
{
    memset(out, 0, 16);
    for (int p = 0; p < 128; p++)
        if ((in[p >> 3] >> (p & 7)) & 1) {
            int q = 127 - p;
            out[q >> 3] |= (uint8_t)(1u << (q & 7));
        }
}

/* -------------------------------------------------------- quant ranges ---- */

/* The 21 BISE ranges, in the order the spec enumerates them. */
static const int LEVELS[21] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32,
                               40, 48, 64, 80, 96, 128, 160, 192, 256};

static void range_shape(int q, int *trits, int *quints, int *bits)
{
    int n = LEVELS[q];
    *trits = *quints = 0;
    if (n % 3 == 0) { *trits = 1; n /= 3; }
    else if (n % 5 == 0) { *quints = 1; n /= 5; }
    int b = 0;
    while ((1 << b) < n) b++;
    *bits = b;
}

static int bise_bits(int count, int q)
{
    int t, qu, b;
    range_shape(q, &t, &qu, &b);
    int n = count * b;
    if (t) n += (count * 8 + 4) / 5;
    if (qu) n += (count * 7 + 2) / 3;
    return n;
}

/* Trit block decode: 8 bits T -> 5 trits (spec procedure). */
static void decode_trits(int T, int t[5])
{
    int C;
#define BIT(x, i) (((x) >> (i)) & 1)
    if (((T >> 2) & 7) == 7) {
        C = (((T >> 5) & 7) << 2) | (T & 3);
        t[4] = 2; t[3] = 2;
    } else {
        C = T & 0x1F;
        if (((T >> 5) & 3) == 3) { t[4] = 2; t[3] = BIT(T, 7); }
        else { t[4] = BIT(T, 7); t[3] = (T >> 5) & 3; }
    }
    if ((C & 3) == 3) {
        t[2] = 2; t[1] = BIT(C, 4);
        t[0] = (BIT(C, 3) << 1) | (BIT(C, 2) & !BIT(C, 3));
    } else if (((C >> 2) & 3) == 3) {
        t[2] = 2; t[1] = 2; t[0] = C & 3;
    } else {
        t[2] = BIT(C, 4); t[1] = (C >> 2) & 3;
        t[0] = (BIT(C, 1) << 1) | (BIT(C, 0) & !BIT(C, 1));
    }
}

/* Quint block decode: 7 bits Q -> 3 quints (spec procedure). */
static void decode_quints(int Q, int q[3])
{
    int C;
    if (((Q >> 1) & 3) == 3 && ((Q >> 5) & 3) == 0) {
        q[2] = (BIT(Q, 0) << 2) | ((BIT(Q, 4) & !BIT(Q, 0)) << 1) | (BIT(Q, 3) & !BIT(Q, 0));
        q[1] = 4; q[0] = 4;
        return;
    }
    if (((Q >> 1) & 3) == 3) {
        q[2] = 4;
        C = (((Q >> 3) & 3) << 3) | ((~(Q >> 5) & 3) << 1) | (Q & 1);
    } else {
        q[2] = (Q >> 5) & 3;
        C = Q & 0x1F;
    }
    if ((C & 7) == 5) { q[1] = 4; q[0] = (C >> 3) & 3; }
    else { q[1] = (C >> 3) & 3; q[0] = C & 7; }
#undef BIT
}

/* Decode `count` BISE integers of range q from a 128-bit buffer starting at
 * bit `start`; only `bise_bits(count,q)` bits belong to the stream and bits
 * past its end read as zero. */
static void bise_decode(const uint8_t *buf, int start, int count, int q, int *out)
{
    int t, qu, b;
    range_shape(q, &t, &qu, &b);
    int total = bise_bits(count, q);
    uint8_t s[32];
    memset(s, 0, sizeof s);
    for (int i = 0; i < total; i++)
        if (rd(buf, start + i, 1)) s[i >> 3] |= (uint8_t)(1u << (i & 7));
    int pos = 0;
    if (t) {
        for (int g = 0; g < count; g += 5) {
            int m[5], T = 0;
            static const int tb[5] = {2, 2, 1, 2, 1};
            int tshift = 0;
            for (int j = 0; j < 5; j++) {
                m[j] = (int)rd(s, pos, b); pos += b;
                T |= (int)rd(s, pos, tb[j]) << tshift; pos += tb[j]; tshift += tb[j];
            }
            int d[5];
            decode_trits(T, d);
            for (int j = 0; j < 5 && g + j < count; j++) out[g + j] = (d[j] << b) | m[j];
        }
    } else if (qu) {
        for (int g = 0; g < count; g += 3) {
            int m[3], Q = 0;
            static const int qb[3] = {3, 2, 2};
            int qshift = 0;
            for (int j = 0; j < 3; j++) {
                m[j] = (int)rd(s, pos, b); pos += b;
                Q |= (int)rd(s, pos, qb[j]) << qshift; pos += qb[j]; qshift += qb[j];
            }
            int d[3];
            decode_quints(Q, d);
            for (int j = 0; j < 3 && g + j < count; j++) out[g + j] = (d[j] << b) | m[j];
        }
    } else {
        for (int i = 0; i < count; i++) { out[i] = (int)rd(s, pos, b); pos += b; }
    }
}

/* ------------------------------------------------------ unquantisation ---- */

/* Replicate the low `bits` bits of v up to `to` bits. */
static int replicate(int v, int bits, int to)
{
    if (bits == 0) return 0;
    int r = 0, have = 0;
    while (have < to) {
        int take = bits < (to - have) ? bits : (to - have);
        r = (r << take) | (v >> (bits - take));
        have += take;
    }
    return r;
}

/* Colour value unquantisation to 0..255 (spec table "Color Unquantization"). */
static int unq_color(int q, int v)
{
    int t, qu, b;
    range_shape(q, &t, &qu, &b);
    if (!t && !qu) return replicate(v, b, 8);
    int D = v >> b, m = v & ((1 << b) - 1);
    int a = m & 1, bb = (m >> 1) & 1, c = (m >> 2) & 1, d = (m >> 3) & 1, e = (m >> 4) & 1, f = (m >> 5) & 1;
    int A = a ? 0x1FF : 0, B = 0, C = 0;
    int L = LEVELS[q];
    switch (L) {
    case 6:   B = 0; C = 204; break;
    case 10:  B = 0; C = 113; break;
    case 12:  B = (bb << 8) | (bb << 4) | (bb << 2) | (bb << 1); C = 93; break;
    case 20:  B = (bb << 8) | (bb << 3) | (bb << 2); C = 54; break;
    case 24:  B = (c << 8) | (bb << 7) | (c << 3) | (bb << 2) | (c << 1) | bb; C = 44; break;
    case 40:  B = (c << 8) | (bb << 7) | (c << 2) | (bb << 1) | c; C = 26; break;
    case 48:  B = (d << 8) | (c << 7) | (bb << 6) | (d << 2) | (c << 1) | bb; C = 22; break;
    case 80:  B = (d << 8) | (c << 7) | (bb << 6) | (d << 1) | c; C = 13; break;
    case 96:  B = (e << 8) | (d << 7) | (c << 6) | (bb << 5) | (e << 1) | d; C = 11; break;
    case 160: B = (e << 8) | (d << 7) | (c << 6) | (bb << 5) | e; C = 6; break;
    case 192: B = (f << 8) | (e << 7) | (d << 6) | (c << 5) | (bb << 4) | f; C = 5; break;
    default:  return -1; /* ranges 3 and 5 never carry colour values */
    }
    int T = D * C + B;
    T ^= A;
    return (A & 0x80) | (T >> 2);
}

/* Weight unquantisation to 0..64 (spec table "Weight Unquantization"). */
static int unq_weight(int q, int v)
{
    int t, qu, b;
    range_shape(q, &t, &qu, &b);
    int r;
    if (!t && !qu) {
        r = replicate(v, b, 6);
    } else if (b == 0) {
        static const int w3[3] = {0, 32, 63}, w5[5] = {0, 16, 32, 47, 63};
        r = t ? w3[v] : w5[v];
    } else {
        int D = v >> b, m = v & ((1 << b) - 1);
        int a = m & 1, bb = (m >> 1) & 1, c = (m >> 2) & 1;
        int A = a ? 0x7F : 0, B = 0, C = 0;
        switch (LEVELS[q]) {
        case 6:  B = 0; C = 50; break;
        case 10: B = 0; C = 28; break;
        case 12: B = (bb << 6) | (bb << 2) | bb; C = 23; break;
        case 20: B = (bb << 6) | (bb << 1); C = 13; break;
        case 24: B = (c << 6) | (bb << 5) | (c << 1) | bb; C = 11; break;
        default: return -1;
        }
        int T = D * C + B;
        T ^= A;
        r = (A & 0x20) | (T >> 2);
    }
    if (r > 32) r++;
    return r;
}

/* ------------------------------------------------------ partition hash ---- */

static uint32_t hash52(uint32_t p)
{
    p ^= p >> 15;
    p *= 0xEEDE0891u;
    p ^= p >> 5;
    p += p << 16;
    p ^= p >> 7;
    p ^= p >> 3;
    p ^= p << 6;
    p ^= p >> 17;
    return p;
}

static int select_partition(int seed, int x, int y, int z, int count, int small)
{
    if (small) { x <<= 1; y <<= 1; z <<= 1; }
    seed += (count - 1) * 1024;
    uint32_t r = hash52((uint32_t)seed);
    uint32_t s[12];
    s[0] = r & 0xF;          s[1] = (r >> 4) & 0xF;   s[2] = (r >> 8) & 0xF;
    s[3] = (r >> 12) & 0xF;  s[4] = (r >> 16) & 0xF;  s[5] = (r >> 20) & 0xF;
    s[6] = (r >> 24) & 0xF;  s[7] = (r >> 28) & 0xF;  s[8] = (r >> 18) & 0xF;
    s[9] = (r >> 22) & 0xF;  s[10] = (r >> 26) & 0xF; s[11] = ((r >> 30) | (r << 2)) & 0xF;
    for (int i = 0; i < 12; i++) s[i] *= s[i];
    int sh1, sh2;
    if (seed & 1) { sh1 = (seed & 2) ? 4 : 5; sh2 = (count == 3) ? 6 : 5; }
    else { sh1 = (count == 3) ? 6 : 5; sh2 = (seed & 2) ? 4 : 5; }
    int sh3 = (seed & 0x10) ? sh1 : sh2;
    s[0] >>= sh1; s[1] >>= sh2; s[2] >>= sh1; s[3] >>= sh2;
    s[4] >>= sh1; s[5] >>= sh2; s[6] >>= sh1; s[7] >>= sh2;
    s[8] >>= sh3; s[9] >>= sh3; s[10] >>= sh3; s[11] >>= sh3;
    int a = (int)((s[0] * x + s[1] * y + s[10] * z + (r >> 14)) & 0x3F);
    int b = (int)((s[2] * x + s[3] * y + s[11] * z + (r >> 10)) & 0x3F);
    int c = (int)((s[4] * x + s[5] * y + s[8] * z + (r >> 6)) & 0x3F);
    int d = (int)((s[6] * x + s[7] * y + s[9] * z + (r >> 2)) & 0x3F);
    if (count < 4) d = 0;
    if (count < 3) c = 0;
    if (a >= b && a >= c && a >= d) return 0;
    if (b >= c && b >= d) return 1;
    if (c >= d) return 2;
    return 3;
}

/* ------------------------------------------------------ endpoint modes ---- */

static int clamp255(int v) { return v < 0 ? 0 : (v > 255 ? 255 : v); }

static void bit_transfer_signed(int *a, int *b)
{
    *b >>= 1;
    *b |= *a & 0x80;
    *a >>= 1;
    *a &= 0x3F;
    if (*a & 0x20) *a -= 0x40;
}

static void blue_contract(int c[4])
{
    c[0] = (c[0] + c[2]) >> 1;
    c[1] = (c[1] + c[2]) >> 1;
}

/* Returns 0 on success, 1 for an HDR mode (an error in the LDR profile). */
static int decode_endpoints(int cem, const int *v, int e0[4], int e1[4])
{
    int a, b, c, d, s0, s1, v0, v1, v2, v3, v4, v5, v6, v7;
    switch (cem) {
    case 0:
        e0[0] = e0[1] = e0[2] = v[0]; e0[3] = 255;
        e1[0] = e1[1] = e1[2] = v[1]; e1[3] = 255;
        return 0;
    case 1: {
        int l0 = (v[0] >> 2) | (v[1] & 0xC0);
        int l1 = l0 + (v[1] & 0x3F);
        if (l1 > 255) l1 = 255;
        e0[0] = e0[1] = e0[2] = l0; e0[3] = 255;
        e1[0] = e1[1] = e1[2] = l1; e1[3] = 255;
        return 0;
    }
    case 4:
        e0[0] = e0[1] = e0[2] = v[0]; e0[3] = v[2];
        e1[0] = e1[1] = e1[2] = v[1]; e1[3] = v[3];
        return 0;
    case 5:
        v0 = v[0]; v1 = v[1]; v2 = v[2]; v3 = v[3];
        bit_transfer_signed(&v1, &v0);
        bit_transfer_signed(&v3, &v2);
        e0[0] = e0[1] = e0[2] = v0; e0[3] = v2;
        e1[0] = e1[1] = e1[2] = clamp255(v0 + v1); e1[3] = clamp255(v2 + v3);
        return 0;
    case 6:
        e0[0] = (v[0] * v[3]) >> 8; e0[1] = (v[1] * v[3]) >> 8; e0[2] = (v[2] * v[3]) >> 8; e0[3] = 255;
        e1[0] = v[0]; e1[1] = v[1]; e1[2] = v[2]; e1[3] = 255;
        return 0;
    case 8:
    case 12:
        s0 = v[0] + v[2] + v[4];
        s1 = v[1] + v[3] + v[5];
        a = (cem == 12) ? v[6] : 255;
        b = (cem == 12) ? v[7] : 255;
        if (s1 >= s0) {
            e0[0] = v[0]; e0[1] = v[2]; e0[2] = v[4]; e0[3] = a;
            e1[0] = v[1]; e1[1] = v[3]; e1[2] = v[5]; e1[3] = b;
        } else {
            e0[0] = v[1]; e0[1] = v[3]; e0[2] = v[5]; e0[3] = b;
            e1[0] = v[0]; e1[1] = v[2]; e1[2] = v[4]; e1[3] = a;
            blue_contract(e0);
            blue_contract(e1);
        }
        return 0;
    case 9:
    case 13:
        v0 = v[0]; v1 = v[1]; v2 = v[2]; v3 = v[3]; v4 = v[4]; v5 = v[5];
        v6 = (cem == 13) ? v[6] : 255; v7 = (cem == 13) ? v[7] : 0;
        bit_transfer_signed(&v1, &v0);
        bit_transfer_signed(&v3, &v2);
        bit_transfer_signed(&v5, &v4);
        if (cem == 13) bit_transfer_signed(&v7, &v6);
        if (v1 + v3 + v5 >= 0) {
            e0[0] = v0; e0[1] = v2; e0[2] = v4; e0[3] = v6;
            e1[0] = v0 + v1; e1[1] = v2 + v3; e1[2] = v4 + v5; e1[3] = v6 + v7;
        } else {
            e0[0] = v0 + v1; e0[1] = v2 + v3; e0[2] = v4 + v5; e0[3] = v6 + v7;
            e1[0] = v0; e1[1] = v2; e1[2] = v4; e1[3] = v6;
            blue_contract(e0);
            blue_contract(e1);
        }
        for (c = 0; c < 4; c++) { e0[c] = clamp255(e0[c]); e1[c] = clamp255(e1[c]); }
        return 0;
    case 10:
        e0[0] = (v[0] * v[3]) >> 8; e0[1] = (v[1] * v[3]) >> 8; e0[2] = (v[2] * v[3]) >> 8; e0[3] = v[4];
        e1[0] = v[0]; e1[1] = v[1]; e1[2] = v[2]; e1[3] = v[5];
        return 0;
    default:
        (void)d;
        return 1;
    }
}

/* ----------------------------------------------------------- block mode --- */

typedef struct {
    int wx, wy, dual, wq; /* weight grid, dual plane flag, weight range index */
} mode_t_;

/* Returns 0 when the 11-bit mode is a normal (non-reserved) 2D block mode. */
static int decode_block_mode(int m, mode_t_ *o)
{
    int R, H = (m >> 9) & 1, D = (m >> 10) & 1;
    int A = (m >> 5) & 3, B = (m >> 7) & 3;
    if (m & 3) {
        R = ((m & 3) << 1) | ((m >> 4) & 1);
        switch ((m >> 2) & 3) {
        case 0: o->wx = B + 4; o->wy = A + 2; break;
        case 1: o->wx = B + 8; o->wy = A + 2; break;
        case 2: o->wx = A + 2; o->wy = B + 8; break;
        default:
            if ((m >> 8) & 1) { o->wx = (B & 1) + 2; o->wy = A + 2; }
            else { o->wx = A + 2; o->wy = (B & 1) + 6; }
            break;
        }
    } else {
        R = (((m >> 2) & 3) << 1) | ((m >> 4) & 1);
        if (((m >> 2) & 3) == 0) return 1; /* reserved */
        switch ((m >> 7) & 3) {
        case 0: o->wx = 12; o->wy = A + 2; break;
        case 1: o->wx = A + 2; o->wy = 12; break;
        case 2: o->wx = A + 6; o->wy = ((m >> 9) & 3) + 6; H = 0; D = 0; break;
        default:
            if (A == 0) { o->wx = 6; o->wy = 10; }
            else if (A == 1) { o->wx = 10; o->wy = 6; }
            else return 1; /* reserved (the void-extent pattern is handled earlier) */
            break;
        }
    }
    /* R in 2..7 selects the range; H adds 6 (spec weight-range table). */
    o->wq = (R - 2) + 6 * H;
    o->dual = D;
    return 0;
}

/* ----------------------------------------------------------- the decoder -- */

/*
 * Decode one block of footprint bx x by (2D). `c16` receives bx*by texels x 4
 * channels of UNORM16 values, texel order row-major (y * bx + x).
 * Returns AO_OK, AO_ERROR_BLOCK (error colour written) or AO_VOID_EXTENT.
 */
int astc_oracle_decode_block(const uint8_t *blk, int bx, int by, uint16_t *c16)
{
    int n = bx * by;
    int mode = (int)rd(blk, 0, 11);
#define ERR() do { for (int i_ = 0; i_ < n; i_++) { c16[4*i_] = 0xFFFF; c16[4*i_+1] = 0; c16[4*i_+2] = 0xFFFF; c16[4*i_+3] = 0xFFFF; } return AO_ERROR_BLOCK; } while (0)

    if ((mode & 0x1FF) == 0x1FC) {
        if ((mode >> 9) & 1) ERR();            /* HDR void extent in LDR profile */
        if (rd(blk, 10, 2) != 3) ERR();        /* reserved bits 10..11 must be 1 */
        uint32_t s0 = rd(blk, 12, 13), s1 = rd(blk, 25, 13), t0 = rd(blk, 38, 13), t1 = rd(blk, 51, 13);
        int all_ones = s0 == 0x1FFF && s1 == 0x1FFF && t0 == 0x1FFF && t1 == 0x1FFF;
        if (!all_ones && (s0 >= s1 || t0 >= t1)) ERR();
        for (int i = 0; i < n; i++)
            for (int c = 0; c < 4; c++) c16[4 * i + c] = (uint16_t)rd(blk, 64 + 16 * c, 16);
        return AO_VOID_EXTENT;
    }

    mode_t_ bm;
    if (decode_block_mode(mode, &bm)) ERR();
    int nweights = bm.wx * bm.wy * (bm.dual + 1);
    if (nweights > 64) ERR();
    if (bm.wx > bx || bm.wy > by) ERR();
    int wbits = bise_bits(nweights, bm.wq);
    if (wbits < 24 || wbits > 96) ERR();

    int parts = (int)rd(blk, 11, 2) + 1;
    if (bm.dual && parts == 4) ERR();

    int cem[4], seed = 0, color_start, extra = 0;
    int below = 128 - wbits - (bm.dual ? 2 : 0); /* first bit above the colour area */
    if (parts == 1) {
        cem[0] = (int)rd(blk, 13, 4);
        color_start = 17;
    } else {
        seed = (int)rd(blk, 13, 10);
        int field = (int)rd(blk, 23, 6);
        color_start = 29;
        if ((field & 3) == 0) {
            for (int p = 0; p < parts; p++) cem[p] = field >> 2;
        } else {
            extra = 3 * parts - 4;
            int hi = (int)rd(blk, below - extra, extra);
            int all = (field >> 2) | (hi << 4);
            int base = (field & 3) - 1;
            for (int p = 0; p < parts; p++) {
                int cbit = (all >> p) & 1;
                int mbits = (all >> (parts + 2 * p)) & 3;
                cem[p] = ((base + cbit) << 2) | mbits;
            }
        }
    }
    int nints = 0;
    for (int p = 0; p < parts; p++) nints += 2 * ((cem[p] >> 2) + 1);
    if (nints > 18) ERR();
    int avail = below - extra - color_start;
    int cq = -1;
    for (int q = 20; q >= 4; q--)
        if (bise_bits(nints, q) <= avail) { cq = q; break; }
    if (cq < 0) ERR();

    int raw[18], col[18];
    bise_decode(blk, color_start, nints, cq, raw);
    for (int i = 0; i < nints; i++) col[i] = unq_color(cq, raw[i]);

    int e0[4][4], e1[4][4];
    for (int p = 0, k = 0; p < parts; p++) {
        if (decode_endpoints(cem[p], col + k, e0[p], e1[p])) ERR(); /* HDR mode */
        k += 2 * ((cem[p] >> 2) + 1);
    }

    uint8_t rev[16];
    reverse128(blk, rev);
    int wraw[64], w[64];
    bise_decode(rev, 0, nweights, bm.wq, wraw);
    for (int i = 0; i < nweights; i++) w[i] = unq_weight(bm.wq, wraw[i]);
    int ccs = bm.dual ? (int)rd(blk, 128 - wbits - 2, 2) : -1;

    int ds = (1024 + bx / 2) / (bx - 1);
    int dt = (1024 + by / 2) / (by - 1);
    int planes = bm.dual + 1;
    int small = n < 31;
    for (int y = 0; y < by; y++)
        for (int x = 0; x < bx; x++) {
            int pw[2];
            int gs = (ds * x * (bm.wx - 1) + 32) >> 6;
            int gt = (dt * y * (bm.wy - 1) + 32) >> 6;
            int js = gs >> 4, fs = gs & 15, jt = gt >> 4, ft = gt & 15;
            int w11 = (fs * ft + 8) >> 4;
            int w10 = ft - w11, w01 = fs - w11, w00 = 16 - fs - ft + w11;
            for (int pl = 0; pl < planes; pl++) {
                int v0 = js + jt * bm.wx;
                int p00 = w[v0 * planes + pl];
                int p01 = (js + 1 < bm.wx) ? w[(v0 + 1) * planes + pl] : 0;
                int p10 = (jt + 1 < bm.wy) ? w[(v0 + bm.wx) * planes + pl] : 0;
                int p11 = (js + 1 < bm.wx && jt + 1 < bm.wy) ? w[(v0 + bm.wx + 1) * planes + pl] : 0;
                pw[pl] = (p00 * w00 + p01 * w01 + p10 * w10 + p11 * w11 + 8) >> 4;
            }
            int part = parts > 1 ? select_partition(seed, x, y, 0, parts, small) : 0;
            for (int c = 0; c < 4; c++) {
                int wt = (c == ccs) ? pw[1] : pw[0];
                int c0 = e0[part][c] * 257, c1 = e1[part][c] * 257;
                c16[4 * (y * bx + x) + c] = (uint16_t)((c0 * (64 - wt) + c1 * wt + 32) >> 6);
            }
        }
    return AO_OK;
#undef ERR
}

/* UNORM16 -> fp16 bits under the decode_float16 rule for LDR values:
 * 65535 -> 1.0, otherwise C/65536 rounded toward zero. */
uint16_t astc_oracle_unorm16_to_half(uint16_t c)
{
    if (c == 0xFFFF) return 0x3C00;
    if (c < 4) return (uint16_t)(c << 8);           /* subnormal: C * 2^-16 = (256C) * 2^-24 */
    int n = 31 - __builtin_clz((unsigned)c);         /* 2 <= n <= 15 */
    int mant = n >= 10 ? (c >> (n - 10)) : (c << (10 - n));
    return (uint16_t)(((n - 1) << 10) | (mant & 0x3FF));
}

/* ------------------------------------------------------ bulk entry points - */

/* Output modes shared with the CUDA library's decode entry point. */
#define AO_OUT_UNORM8 0
#define AO_OUT_FP16 1
#define AO_OUT_UNORM16 2

typedef struct {
    const uint8_t *blocks;
    int64_t begin, end;
    int bx, by, mode;
    void *out;
} job_t;

static void *run_job(void *arg)
{
    job_t *j = (job_t *)arg;
    int n = j->bx * j->by;
    uint16_t c16[144 * 4];
    for (int64_t i = j->begin; i < j->end; i++) {
        astc_oracle_decode_block(j->blocks + 16 * i, j->bx, j->by, c16);
        if (j->mode == AO_OUT_UNORM8) {
            uint8_t *o = (uint8_t *)j->out + (size_t)i * n * 4;
            for (int k = 0; k < 4 * n; k++) o[k] = (uint8_t)(c16[k] >> 8);
        } else if (j->mode == AO_OUT_FP16) {
            uint16_t *o = (uint16_t *)j->out + (size_t)i * n * 4;
            for (int k = 0; k < 4 * n; k++) o[k] = astc_oracle_unorm16_to_half(c16[k]);
        } else {
            uint16_t *o = (uint16_t *)j->out + (size_t)i * n * 4;
            memcpy(o, c16, sizeof(uint16_t) * 4 * n);
        }
    }
    return NULL;
}

/*
 * Decode `nblocks` consecutive blocks into per-block texel arrays
 * out[block][y][x][rgba] (the same layout as the CUDA decode entry point).
 * mode: 0 = UNORM8, 1 = fp16 bits, 2 = UNORM16. Returns 0, or -1 on bad args.
 */
int astc_oracle_decode_blocks(const uint8_t *blocks, int64_t nblocks, int bx, int by,
                              int mode, void *out, int threads)
{
    if (!blocks || !out || nblocks < 0 || bx < 4 || by < 4 || bx > 12 || by > 12 || mode < 0 || mode > 2)
        return -1;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((int64_t)threads > nblocks) threads = nblocks > 0 ? (int)nblocks : 1;
    job_t jobs[256];
    pthread_t tid[256];
    for (int t = 0; t < threads; t++) {
        jobs[t].blocks = blocks;
        jobs[t].begin = nblocks * t / threads;
        jobs[t].end = nblocks * (t + 1) / threads;
        jobs[t].bx = bx; jobs[t].by = by; jobs[t].mode = mode; jobs[t].out = out;
    }
    for (int t = 1; t < threads; t++) pthread_create(&tid[t], NULL, run_job, &jobs[t]);
    run_job(&jobs[0]);
    for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
    return 0;
}

/*
 * Image-level decode with the shape of the reference's `akv_decode`
 * (astc_kv/bridge.cpp:27-35): blocks in row-major block order for a w x h
 * image, output float32 RGBA h x w x 4 holding the fp16 view of each texel.
 */
int astc_oracle_decode_image_f32(const uint8_t *blocks, size_t bytes, int bx, int by,
                                 float *rgba, unsigned w, unsigned h)
{
    int cols = (int)((w + bx - 1) / bx), rows = (int)((h + by - 1) / by);
    if ((size_t)cols * rows * 16 != bytes) return -1;
    uint16_t c16[144 * 4];
    for (int r = 0; r < rows; r++)
        for (int c = 0; c < cols; c++) {
            astc_oracle_decode_block(blocks + 16 * ((size_t)r * cols + c), bx, by, c16);
            for (int y = 0; y < by; y++)
                for (int x = 0; x < bx; x++) {
                    unsigned px = (unsigned)(c * bx + x), py = (unsigned)(r * by + y);
                    if (px >= w || py >= h) continue;
                    for (int k = 0; k < 4; k++) {
                        uint16_t hb = astc_oracle_unorm16_to_half(c16[4 * (y * bx + x) + k]);
                        /* exact fp16 -> fp32 widening */
                        uint32_t sign = 0, e = (hb >> 10) & 0x1F, m = hb & 0x3FF, f;
                        if (e == 0) {
                            if (m == 0) f = sign;
                            else { int s = 0; while (!(m & 0x400)) { m <<= 1; s++; } m &= 0x3FF; f = ((uint32_t)(113 - s) << 23) | (m << 13); }
                        } else f = ((e + 112) << 23) | (m << 13);
                        float fv;
                        memcpy(&fv, &f, 4);
                        rgba[((size_t)py * w + px) * 4 + k] = fv;
                    }
                }
        }
    return 0;
}

/* Block statistics for tests: partition count, dual plane, weight grid,
 * weight range, colour range, CEM of partition 0, kind (0 normal, 1 error,
 * 2 void extent). Fills info[8]. */
int astc_oracle_block_info(const uint8_t *blk, int bx, int by, int *info)
{
    uint16_t c16[144 * 4];
    int kind = astc_oracle_decode_block(blk, bx, by, c16);
    memset(info, 0, 8 * sizeof(int));
    info[7] = kind;
    if (kind != AO_OK) return kind;
    int mode = (int)rd(blk, 0, 11);
    mode_t_ bm;
    decode_block_mode(mode, &bm);
    int parts = (int)rd(blk, 11, 2) + 1;
    info[0] = parts; info[1] = bm.dual; info[2] = bm.wx; info[3] = bm.wy; info[4] = bm.wq;
    int nweights = bm.wx * bm.wy * (bm.dual + 1);
    int wbits = bise_bits(nweights, bm.wq);
    int cem0 = parts == 1 ? (int)rd(blk, 13, 4) : -1;
    if (parts > 1) {
        int field = (int)rd(blk, 23, 6);
        if ((field & 3) == 0) cem0 = field >> 2;
        else {
            int extra = 3 * parts - 4, below = 128 - wbits - (bm.dual ? 2 : 0);
            int all = (field >> 2) | ((int)rd(blk, below - extra, extra) << 4);
            cem0 = (((field & 3) - 1 + (all & 1)) << 2) | ((all >> parts) & 3);
        }
    }
    info[6] = cem0;
    (void)wbits;
    return kind;
}

/* Exposed for table self-tests. */
int astc_oracle_unquant_color(int q, int v) { return unq_color(q, v); }
int astc_oracle_unquant_weight(int q, int v) { return unq_weight(q, v); }
int astc_oracle_partition(int seed, int x, int y, int count, int small) { return select_partition(seed, x, y, 0, count, small); }
int astc_oracle_bise_bits(int count, int q) { return bise_bits(count, q); }
