/* CPU restatement of the reference NF4 decoder -- TEST INFRASTRUCTURE.
 *
 * Only the tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library (oracle/_build/libnf4_oracle.so).  The shipped CUDA path never
 * does.
 *
 * Follows solution/kernels/nf4.py:41-59 of the reference:
 *   byte  = packed[i / 2];  nibble = (i even) ? byte >> 4 : byte & 15
 *   scale = fp32(fp32(code2[qabs[i/64]] * absmax2[(i/64)/256]) + offset)   (nested)
 *         = absmax[i/64]                                                   (flat)
 *   out   = fp16_rn(NF4[nibble] * scale)   (fp32 product, one rounding)
 * Compiled with -ffp-contract=off so the multiply and the add are separate
 * IEEE operations, matching the reference's enable_fp_fusion=False.
 * Blocks are split across POSIX threads (the CPU baseline passes the host core count).
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

static const float kNF4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

/* IEEE binary32 -> binary16, round to nearest even, with subnormals, inf, nan. */
static uint16_t f32_to_f16_rn(float value) {
    uint32_t x;
    memcpy(&x, &value, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {                       /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
    }
    int e = (int)exp - 127 + 15;              /* rebiased exponent */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);   /* overflow -> inf */
    if (e <= 0) {                             /* subnormal or zero in fp16 */
        if (e < -10) return (uint16_t)sign;   /* rounds to signed zero */
        uint32_t full = man | 0x800000u;      /* implicit bit */
        int shift = 14 - e;                   /* bits to drop */
        uint32_t kept = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (kept & 1u))) kept += 1u;
        return (uint16_t)(sign | kept);       /* carry into exponent is correct */
    }
    uint32_t kept = man >> 13;
    uint32_t rem = man & 0x1fffu;
    uint32_t out = sign | ((uint32_t)e << 10) | kept;
    if (rem > 0x1000u || (rem == 0x1000u && (kept & 1u))) out += 1u;  /* may carry to inf */
    return (uint16_t)out;
}

static inline int nibble_at(const uint8_t* packed, int64_t i) {
    uint8_t b = packed[i >> 1];
    return (i & 1) ? (b & 15) : (b >> 4);
}

typedef struct {
    const uint8_t* packed; const uint8_t* qabs; const float* absmax2; const float* code2;
    const float* flat_absmax; float offset; uint16_t* out; int64_t n; int64_t b0, b1;
} job_t;

static void* run_job(void* arg) {
    job_t* j = (job_t*)arg;
    for (int64_t b = j->b0; b < j->b1; ++b) {
        float scale;
        if (j->flat_absmax) {
            scale = j->flat_absmax[b];
        } else {
            volatile float decoded = j->code2[j->qabs[b]] * j->absmax2[b >> 8];
            scale = decoded + j->offset;
        }
        int64_t end = (b + 1) * 64 < j->n ? (b + 1) * 64 : j->n;
        for (int64_t i = b * 64; i < end; ++i) {
            j->out[i] = f32_to_f16_rn(kNF4[nibble_at(j->packed, i)] * scale);
        }
    }
    return 0;
}

static int run_all(job_t proto, int threads) {
    int64_t blocks = (proto.n + 63) / 64;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((int64_t)threads > blocks) threads = blocks > 0 ? (int)blocks : 1;
    pthread_t tid[256];
    job_t jobs[256];
    int spawned[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = proto;
        jobs[t].b0 = blocks * t / threads;
        jobs[t].b1 = blocks * (t + 1) / threads;
        spawned[t] = t != threads - 1 && pthread_create(&tid[t], 0, run_job, &jobs[t]) == 0;
        if (!spawned[t]) run_job(&jobs[t]);   /* last slice (or a failed spawn) runs inline */
    }
    for (int t = 0; t < threads; ++t) {
        if (spawned[t]) pthread_join(tid[t], 0);
    }
    return 0;
}

int nf4_oracle_dequant_nested(const uint8_t* packed, const uint8_t* qabs, const float* absmax2,
                              const float* code2, float offset, uint16_t* out, int64_t n,
                              int threads) {
    job_t j = {packed, qabs, absmax2, code2, 0, offset, out, n, 0, 0};
    return run_all(j, threads);
}

int nf4_oracle_dequant_flat(const uint8_t* packed, const float* absmax, uint16_t* out, int64_t n,
                            int threads) {
    job_t j = {packed, 0, 0, 0, absmax, 0.0f, out, n, 0, 0};
    return run_all(j, threads);
}

uint16_t nf4_oracle_f32_to_f16(float value) { return f32_to_f16_rn(value); }
