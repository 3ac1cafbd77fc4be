/* harness_common.h -- host/B200 variant of the corpus harness header.
 *
 * The corpus's per-kernel harness.c files include "harness_common.h" and use
 * the names below (env/harness/harness_common.h of sriharshapy/hexkernels).
 * This header keeps those names and meanings so each harness.c compiles
 * unchanged on an x86 host and links against a candidate_kernel that runs on
 * a B200 through libhexcuda (or against the CPU oracle):
 *
 *  - HVX_TIME_KERNEL(OUT, STMT): OUT receives the wall-clock nanoseconds of
 *    STMT (host CLOCK_MONOTONIC; the Hexagon pcycle counter does not exist
 *    here).  When libhexcuda is linked, the device time of the last launch,
 *    measured with a cudaEvent pair on the launching stream, is printed as
 *    "HEXCUDA_KERNEL_US kernel=<device us> wall=<call us> launches=<n>" (n =
 *    libhexcuda kernel launches made by STMT).
 *  - hvx_lcg, hvx_report, hvx_report_u16, hvx_close_f32, hvx_close_f16bits:
 *    same arithmetic and output line format (HVXENV_CORRECT / HVXENV_INCORRECT)
 *    as the corpus, so the corpus's evaluate.py result parser still applies.
 *  - HMX / VTCM helpers: the Hexagon context switch is a no-op; layout helpers
 *    keep their index formulas (they are plain integer maps).
 *
 * Compile harnesses with -D__fp16=_Float16 (x86 gcc spells binary16 that way).
 */
#ifndef HVX_HARNESS_COMMON_H
#define HVX_HARNESS_COMMON_H

#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#define HVX_ALIGN __attribute__((aligned(128)))

/* libhexcuda's device-time query; weak so a harness linked against the CPU
 * oracle (no libhexcuda) still links and simply prints no device time. */
extern float hexcuda_last_kernel_ms(void) __attribute__((weak));
extern uint64_t hexcuda_launch_count(void) __attribute__((weak));
extern unsigned hexcuda_mechanisms(int reset) __attribute__((weak));

static inline void hvx_enable_pcycle(void) {}
static inline unsigned long long hvx_rdpcyc(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (unsigned long long)ts.tv_sec * 1000000000ull + (unsigned long long)ts.tv_nsec;
}

#define HVX_TIME_KERNEL(OUT, STMT) do {                                        \
    unsigned long long _hx_l0 = hexcuda_launch_count ? hexcuda_launch_count() : 0; \
    if (hexcuda_mechanisms) hexcuda_mechanisms(1);                             \
    unsigned long long _hx_t0 = hvx_rdpcyc();                                  \
    STMT;                                                                      \
    unsigned long long _hx_t1 = hvx_rdpcyc();                                  \
    (OUT) = _hx_t1 - _hx_t0;                                                   \
    if (hexcuda_last_kernel_ms)                                                \
        printf("HEXCUDA_KERNEL_US kernel=%.3f wall=%.3f launches=%llu mech=0x%x\n", \
               1000.0 * (double)hexcuda_last_kernel_ms(),                      \
               (double)(OUT) / 1000.0,                                         \
               (hexcuda_launch_count ? hexcuda_launch_count() : 0) - _hx_l0,   \
               hexcuda_mechanisms ? hexcuda_mechanisms(0) : 0u);               \
} while (0)

/* LCG: s = s * 1664525 + 1013904223 (mod 2^32), as the corpus harnesses use. */
static inline uint32_t hvx_lcg(uint32_t *s) {
    *s = (*s) * 1664525u + 1013904223u;
    return *s;
}

static inline void hvx_report(int errors, int n, int first_bad, long got, long exp) {
    if (errors == 0)
        printf("HVXENV_CORRECT errors=0 n=%d\n", n);
    else
        printf("HVXENV_INCORRECT errors=%d n=%d first_bad=%d got=%ld exp=%ld\n",
               errors, n, first_bad, got, exp);
}
static inline void hvx_report_u16(int errors, int n, int first_bad,
                                  unsigned short got, unsigned short exp) {
    hvx_report(errors, n, first_bad, (long)got, (long)exp);
}

/* VTCM and HMX do not exist on this target; the base is kept only so code that
 * names it compiles.  Nothing here dereferences it. */
#define HVX_VTCM_BASE 0u
static inline void hvx_hmx_enable(void) {}

/* Layout maps (pure integer index formulas of the corpus's 32x32 tiles). */
static inline int hvx_crouton_off(int r, int c) { return (r / 2) * 64 + c * 2 + (r & 1); }
static inline int hvx_hmx_i8_act_off(int i, int k) { return 2 * hvx_crouton_off(i, k) + 1; }
static inline int hvx_hmx_i8_wgt_off(int k, int j) { return (k / 4) * 128 + j * 4 + (k % 4); }
static inline int hvx_hmx_i8_out_off(int i, int j) { return hvx_crouton_off(i, j); }
static inline int hvx_hmx_requant_0x40(int acc) { return ((acc * 17 + 8) >> 4) & 0xFFF; }

/* Floating-point tolerance compares: |g - e| <= ATOL + RTOL * |e|. */
#ifndef HVX_FP32_ATOL
#define HVX_FP32_ATOL 1e-4f
#endif
#ifndef HVX_FP32_RTOL
#define HVX_FP32_RTOL 1e-3f
#endif
#ifndef HVX_FP16_ATOL
#define HVX_FP16_ATOL 4e-3f
#endif
#ifndef HVX_FP16_RTOL
#define HVX_FP16_RTOL 8e-3f
#endif

static inline int hvx_close_f32(float g, float e) {
    float d = g - e;
    if (d < 0) d = -d;
    float ae = e < 0 ? -e : e;
    return d <= HVX_FP32_ATOL + HVX_FP32_RTOL * ae;
}
static inline int hvx_close_f16bits(unsigned short gb, unsigned short eb) {
    _Float16 gh, eh;
    memcpy(&gh, &gb, 2);
    memcpy(&eh, &eb, 2);
    float g = (float)gh, e = (float)eh, d = g - e;
    if (d < 0) d = -d;
    float ae = e < 0 ? -e : e;
    return d <= HVX_FP16_ATOL + HVX_FP16_RTOL * ae;
}

#endif /* HVX_HARNESS_COMMON_H */
