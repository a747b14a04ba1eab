/* C restatement of the reference harness's input synthesis (TEST INFRASTRUCTURE).
 *
 * Same algorithm as oracle/prng.py, which restates FOG/scripts/fixture_prng.py:44-198
 * (and its Rust mirror FOG/src/bin/test_kernels.rs:34-145). It exists only because the
 * NVFP4 feed-forward weights are 59M elements per matrix and the numpy definition needs
 * several GB of temporaries for them. Only tests, smoke() and bench.py's CPU legs load it.
 */
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <unistd.h>

#define GOLDEN 0x9E3779B97F4A7C15ULL
#define MIX_A 0xBF58476D1CE4E5B9ULL
#define MIX_B 0x94D049BB133111EBULL

static inline uint64_t word_at(uint64_t seed, uint64_t index) {
    /* splitmix64 finaliser applied to (seed ^ index) + golden: fixture_prng.py:57-67 */
    uint64_t x = (seed ^ index) + GOLDEN;
    x = (x ^ (x >> 30)) * MIX_A;
    x = (x ^ (x >> 27)) * MIX_B;
    return x ^ (x >> 31);
}

/* Splits [0, n) into contiguous ranges, one per host thread. */
typedef struct {
    void (*body)(void* ctx, long long lo, long long hi);
    void* ctx;
    long long lo, hi;
} g4o_range;

static void* g4o_run_range(void* arg) {
    g4o_range* r = (g4o_range*)arg;
    r->body(r->ctx, r->lo, r->hi);
    return NULL;
}

static void g4o_parallel(long long n, void (*body)(void*, long long, long long), void* ctx) {
    long threads = sysconf(_SC_NPROCESSORS_ONLN);
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    if (n < (1LL << 16)) threads = 1;
    pthread_t tid[64];
    g4o_range ranges[64];
    long long chunk = (n + threads - 1) / threads;
    int joined[64] = {0};
    for (long t = 0; t < threads; ++t) {
        long long lo = t * chunk < n ? t * chunk : n;
        long long hi = lo + chunk < n ? lo + chunk : n;
        ranges[t] = (g4o_range){body, ctx, lo, hi};
        if (t == 0) continue;
        if (pthread_create(&tid[t], NULL, g4o_run_range, &ranges[t]) == 0)
            joined[t] = 1;
        else
            g4o_run_range(&ranges[t]); /* no thread available: run the range here */
    }
    g4o_run_range(&ranges[0]);
    for (long t = 1; t < threads; ++t)
        if (joined[t]) pthread_join(tid[t], NULL);
}

typedef struct { uint64_t seed; uint8_t* out; } f4_ctx;
static void f4_body(void* c, long long lo, long long hi) {
    f4_ctx* k = (f4_ctx*)c;
    for (long long p = lo; p < hi; ++p) {
        uint8_t a = (uint8_t)((word_at(k->seed, 2 * (uint64_t)p) >> 60) & 0xF);
        uint8_t b = (uint8_t)((word_at(k->seed, 2 * (uint64_t)p + 1) >> 60) & 0xF);
        k->out[p] = (uint8_t)(a | (b << 4));
    }
}

/* e2m1 codes, element 2i in the low nibble of byte i: fixture_prng.py:151-166 */
void g4o_f4_nibbles(uint64_t seed, size_t count, uint8_t* out) {
    f4_ctx k = {seed, out};
    g4o_parallel((long long)(count / 2), f4_body, &k);
}

typedef struct { uint64_t seed, span; int exp_min, is_signed; uint8_t* out; } f8_ctx;
static void f8_body(void* c, long long lo, long long hi) {
    f8_ctx* k = (f8_ctx*)c;
    for (long long i = lo; i < hi; ++i) {
        uint64_t w = word_at(k->seed, (uint64_t)i);
        uint8_t exponent = (uint8_t)(k->exp_min + (int)((w >> 32) % k->span));
        uint8_t mantissa = (uint8_t)((w >> 56) & 0x7);
        uint8_t sign = k->is_signed ? (uint8_t)((w >> 63) << 7) : 0;
        k->out[i] = (uint8_t)(sign | (uint8_t)(exponent << 3) | mantissa);
    }
}

/* e4m3 codes with the exponent field in [exp_min, exp_max]: fixture_prng.py:128-148 */
void g4o_f8_banded(uint64_t seed, size_t count, int exp_min, int exp_max, int is_signed, uint8_t* out) {
    f8_ctx k = {seed, (uint64_t)(exp_max - exp_min + 1), exp_min, is_signed, out};
    g4o_parallel((long long)count, f8_body, &k);
}

/* position-weighted u32 checksum over zero-padded 32-bit words: fixture_prng.py:170-198 */
uint32_t g4o_checksum(const uint8_t* data, size_t nbytes) {
    size_t nwords = (nbytes + 3) / 4;
    uint32_t total = 0;
    for (size_t w = 0; w < nwords; ++w) {
        uint32_t v = 0;
        for (int b = 0; b < 4; ++b) {
            size_t at = w * 4 + (size_t)b;
            if (at < nbytes) v |= (uint32_t)data[at] << (8 * b);
        }
        total += v * ((uint32_t)w * 2u + 1u);
    }
    return total;
}
