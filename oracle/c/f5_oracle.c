/*
 * Plain-C restatement of the W4A8 matvec law -- TEST ORACLE ONLY.
 *
 * This file is test infrastructure: it checks the CUDA product, it is never
 * the thing measured or shipped.  It restates, over a packed DDR row image,
 *
 *   ref/w4a8_ref.py:254-289  matvec_y32  acc_g = sum_{k in g} w*x  (|acc|<2^31)
 *                                        p     = sum_g m_g * acc_g  (int64)
 *                                        y     = rshift_round(p, sh) (|y|<2^31)
 *   ref/w4a8_ref.py:90-99    rshift_round (round half away from zero)
 *   ref/w4a8_ref.py:102-114  row format: K/128 weight beats of 64 B (low
 *                                        nibble = even k), then ceil(NG/32)
 *                                        beats of little-endian uint16 m_g
 *   ref/seq_model.py:431-452 DDRWeights.matvec (the matvec over the image)
 *
 * g = 128 (one beat per group) and g = 64 (two groups per beat) both follow
 * the same per-group sum; integer sums are order-free, so any loop order
 * gives the reference's bit pattern.
 */
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline int64_t rshr64(int64_t v, int s) {
    if (s == 0) return v;
    if (s < 0) return (int64_t)((uint64_t)v << (-s));
    int64_t add = (int64_t)1 << (s - 1);
    return v >= 0 ? (v + add) >> s : -((-v + add) >> s);
}

int f5o_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Returns 0, or -1 if a group accumulator / y32 leaves the range the
 * reference asserts (ref/w4a8_ref.py:285,288). */
int f5o_matvec_rows(const uint8_t *img, long stride, int nrows, int K, int g,
                    const int8_t *x8, int sh, int32_t *y32, int64_t *p_out,
                    int nthreads) {
    const int NG = K / g;
    int bad = 0;
    /* x as int32 once */
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads) reduction(| : bad)
#endif
    for (int r = 0; r < nrows; ++r) {
        const uint8_t *row = img + (long)r * stride;
        const uint8_t *mb = row + K / 2;
        int64_t p = 0;
        for (int gi = 0; gi < NG; ++gi) {
            const uint8_t *wb = row + (long)gi * (g / 2);
            const int8_t *xg = x8 + (long)gi * g;
            int32_t acc = 0;
            for (int j = 0; j < g / 2; ++j) {
                uint8_t b = wb[j];
                int lo = (int)(b & 0xF);
                int hi = (int)(b >> 4);
                lo = lo > 7 ? lo - 16 : lo;
                hi = hi > 7 ? hi - 16 : hi;
                acc += lo * (int)xg[2 * j] + hi * (int)xg[2 * j + 1];
            }
            uint16_t m = (uint16_t)(mb[2 * gi] | ((uint16_t)mb[2 * gi + 1] << 8));
            p += (int64_t)m * (int64_t)acc;
        }
        int64_t y = rshr64(p, sh);
        if (y >= ((int64_t)1 << 31) || y <= -((int64_t)1 << 31)) bad |= 1;
        y32[r] = (int32_t)y;
        if (p_out) p_out[r] = p;
    }
    return bad ? -1 : 0;
}
