/* Host-side model synthesis helpers: seeded normal weights and the GGUF Q8_0 / Q4_K block quantizers.
 *
 * These produce the weight files the library loads (tests and the benchmark have no network for real checkpoints).
 * Block formats (ggml, as GGUF stores them):
 *   Q8_0: per 32 elements  fp16 d, int8 q[32];                    x ~= d * q
 *   Q4_K: per 256 elements fp16 d, fp16 dmin, u8 scales[12], u8 qs[128];
 *         sub-block s (32 elements) has 6-bit sc[s], m[s];       x ~= d*sc[s]*q - dmin*m[s], q in 0..15
 * The quantizers here are this project's own (a min/max fit per sub-block); any quantizer that writes valid blocks
 * is acceptable, because parity is checked against the dequantized values of the bytes actually written.
 * Plain C99 + pthreads; exported symbols are called through ctypes. */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

static uint16_t f32_to_f16(float f) {
  /* round to nearest even, with overflow to inf and gradual underflow */
  uint32_t x; memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t mant = x & 0x7fffffu;
  int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - exp);
    uint32_t half = 1u << (shift - 1);
    uint32_t r = mant >> shift, rem = mant & ((1u << shift) - 1);
    if (rem > half || (rem == half && (r & 1))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t r = mant >> 13, rem = mant & 0x1fffu;
  uint32_t h = sign | ((uint32_t)exp << 10) | r;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) h++;
  return (uint16_t)h;
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ffu, x;
  if (e == 0) {
    if (!m) x = sign;
    else { float f = ldexpf((float)m, -24); memcpy(&x, &f, 4); x |= sign; }
  } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
  else x = sign | ((e + 112) << 23) | (m << 13);
  float f; memcpy(&f, &x, 4); return f;
}

static void q8_0_block(const float *x, uint8_t *out) {
  float amax = 0.f;
  for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
  float d = amax / 127.f;
  uint16_t dh = f32_to_f16(d);
  float id = d > 0 ? 1.f / d : 0.f;
  memcpy(out, &dh, 2);
  for (int i = 0; i < 32; i++) {
    float v = roundf(x[i] * id);
    if (v > 127.f) v = 127.f;
    if (v < -127.f) v = -127.f;
    out[2 + i] = (uint8_t)(int8_t)v;
  }
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

static void q4_k_block(const float *x, uint8_t *out) {
  float scale[8], mins[8], smax = 0.f, mmax = 0.f;
  for (int s = 0; s < 8; s++) {
    float lo = x[32 * s], hi = x[32 * s];
    for (int i = 1; i < 32; i++) { float v = x[32 * s + i]; if (v < lo) lo = v; if (v > hi) hi = v; }
    if (lo > 0.f) lo = 0.f;
    scale[s] = (hi - lo) / 15.f;
    mins[s] = -lo;
    if (scale[s] > smax) smax = scale[s];
    if (mins[s] > mmax) mmax = mins[s];
  }
  uint16_t dh = f32_to_f16(smax / 63.f), mh = f32_to_f16(mmax / 63.f);
  float d = f16_to_f32(dh), dm = f16_to_f32(mh);
  uint8_t sc[8], m[8];
  for (int s = 0; s < 8; s++) {
    sc[s] = (uint8_t)(d > 0 ? clampi((int)lrintf(scale[s] / d), 0, 63) : 0);
    m[s] = (uint8_t)(dm > 0 ? clampi((int)lrintf(mins[s] / dm), 0, 63) : 0);
  }
  memcpy(out, &dh, 2);
  memcpy(out + 2, &mh, 2);
  uint8_t *p = out + 4;
  for (int j = 0; j < 4; j++) {
    p[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    p[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    p[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
  }
  uint8_t q[256];
  for (int s = 0; s < 8; s++) {
    float es = d * (float)sc[s], em = dm * (float)m[s];
    float ie = es > 0 ? 1.f / es : 0.f;
    for (int i = 0; i < 32; i++) q[32 * s + i] = (uint8_t)clampi((int)lrintf((x[32 * s + i] + em) * ie), 0, 15);
  }
  uint8_t *qs = out + 16;
  for (int c = 0; c < 4; c++)
    for (int l = 0; l < 32; l++) qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

typedef struct { const float *x; uint8_t *out; int64_t b0, b1; int kind; } qjob;

static void *qwork(void *a) {
  qjob *j = (qjob *)a;
  for (int64_t b = j->b0; b < j->b1; b++) {
    if (j->kind == 8) q8_0_block(j->x + 32 * b, j->out + 34 * b);
    else q4_k_block(j->x + 256 * b, j->out + 144 * b);
  }
  return 0;
}

static int run_jobs(const float *x, uint8_t *out, int64_t nblocks, int kind, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 64) threads = 64;
  pthread_t th[64]; qjob jb[64];
  int64_t per = (nblocks + threads - 1) / threads;
  int n = 0;
  for (int t = 0; t < threads; t++) {
    int64_t b0 = t * per, b1 = b0 + per < nblocks ? b0 + per : nblocks;
    if (b0 >= b1) break;
    jb[n] = (qjob){x, out, b0, b1, kind};
    if (pthread_create(&th[n], 0, qwork, &jb[n])) { qwork(&jb[n]); continue; }
    n++;
  }
  for (int t = 0; t < n; t++) pthread_join(th[t], 0);
  return 0;
}

/* x: n floats (n % 32 == 0) -> n/32 * 34 bytes */
int synth_quantize_q8_0(const float *x, int64_t n, uint8_t *out, int threads) {
  if (n % 32) return -1;
  return run_jobs(x, out, n / 32, 8, threads);
}

/* x: n floats (n % 256 == 0) -> n/256 * 144 bytes */
int synth_quantize_q4_k(const float *x, int64_t n, uint8_t *out, int threads) {
  if (n % 256) return -1;
  return run_jobs(x, out, n / 256, 12, threads);
}

/* Seeded standard normals scaled by std: a counter-based generator (splitmix64 of seed ^ stream, index) through
 * Box-Muller, so any element range can be produced independently and in parallel. */
static uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

typedef struct { float *x; int64_t i0, i1; uint64_t key; float std; } njob;

static void *nwork(void *a) {
  njob *j = (njob *)a;
  for (int64_t i = j->i0 & ~1LL; i < j->i1; i += 2) {
    uint64_t r1 = splitmix64(j->key + (uint64_t)i), r2 = splitmix64(j->key + (uint64_t)i + 1);
    double u1 = ((r1 >> 11) + 1.0) * (1.0 / 9007199254740993.0), u2 = (r2 >> 11) * (1.0 / 9007199254740992.0);
    double rad = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
    if (i >= j->i0) j->x[i - j->i0] = (float)(rad * cos(th)) * j->std;
    if (i + 1 >= j->i0 && i + 1 < j->i1) j->x[i + 1 - j->i0] = (float)(rad * sin(th)) * j->std;
  }
  return 0;
}

/* x[k] = std * N(0,1) sample number (offset + k) of stream `stream` under `seed`, k < n. */
int synth_normal(float *x, int64_t n, uint64_t seed, uint64_t stream, int64_t offset, float std, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 64) threads = 64;
  uint64_t key = splitmix64(seed * 0x100000001b3ull ^ splitmix64(stream));
  pthread_t th[64]; njob jb[64];
  int64_t per = ((n + threads - 1) / threads + 1) & ~1LL;
  int m = 0;
  for (int t = 0; t < threads; t++) {
    int64_t a = offset + t * per, b = a + per < offset + n ? a + per : offset + n;
    if (a >= b) break;
    jb[m] = (njob){x + (a - offset), a, b, key, std};
    if (pthread_create(&th[m], 0, nwork, &jb[m])) { nwork(&jb[m]); continue; }
    m++;
  }
  for (int t = 0; t < m; t++) pthread_join(th[t], 0);
  return 0;
}
