/*
 * bnbq_oracle.c -- CPU restatement of the reference's quantize / dequantize /
 * NF4-GEMV arithmetic (nshepperd/bitsandbytes-jax 0.2.0, "the reference").
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the parity tests and
 * the benchmark's CPU-baseline leg compare the CUDA kernels against. Nothing in
 * the product (bitsandbytes-jax_b200/) links, loads or calls it.
 *
 * Citations are path:line inside the reference project.
 *
 * Fast-math emulation (src/bnb_jax/kernels/_ptx.py:15-33):
 *   mul.ftz.f32   -> ftz(ftz(a) * ftz(b))          (IEEE RN product, subnormal
 *                                                     inputs/result -> signed 0)
 *   abs.ftz.f32   -> fabsf(ftz(x))
 *   max.ftz.f32   -> fmaxf(ftz(a), ftz(b))         (NaN operand -> the other)
 *   rcp.approx.ftz.f32 -> NOT modelled bit-for-bit. Two modes:
 *     * the caller passes the device's own reciprocals (one per block, taken
 *       from the hardware instruction by bnbq_rcp_approx_ftz); the oracle is
 *       then exact;
 *     * otherwise the oracle uses the correctly rounded 1/m and reports, per
 *       element, whether any reciprocal within +-2 ulp of it (an interval that
 *       contains the PTX ISA's documented error bound for rcp.approx.f32) would
 *       give a different code ("ambiguous").
 * One unpinned corner: whether the hardware flushes a product whose exact value
 * lies just under FLT_MIN but rounds up to FLT_MIN. Here the flush is decided
 * after rounding. No test input reaches that corner.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off). The whole file
 * must be compiled without FMA contraction and without fast-math.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };

/* ------------------------------------------------------------ primitives */

static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float ftz(float v) {
  return (v != 0.0f && fabsf(v) < FLT_MIN) ? copysignf(0.0f, v) : v;
}
static inline float mul_ftz(float a, float b) { return ftz(ftz(a) * ftz(b)); }
static inline float abs_ftz(float x) { return fabsf(ftz(x)); }
static inline float max_ftz(float a, float b) { return fmaxf(ftz(a), ftz(b)); }

/* The NF4 table (kernels/dequantize.py:27-32). */
static const float NF4_TABLE[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

/* The 15 NF4 decision thresholds as float32 bits (kernels/quantize.py:46-50). */
static const uint32_t NF4_THRESHOLD_BITS[15] = {
    0xbf591cd9u, 0xbf1c5270u, 0xbeeb8480u, 0xbeadea76u, 0xbe703cecu,
    0xbe0d38bcu, 0xbd3a7871u, 0x3d22faffu, 0x3df64863u, 0x3e5067e0u,
    0x3e9582d4u, 0x3ec753f9u, 0x3f006d03u, 0x3f248dafu, 0x3f5c89d9u};

static inline float load_elem(int dtype, const void* x, int64_t i) {
  if (dtype == OR_F32) return ((const float*)x)[i];
  if (dtype == OR_F16) return (float)((const _Float16*)x)[i];
  return f32_from_bits((uint32_t)((const uint16_t*)x)[i] << 16);
}

/* cvt.rn.bf16.f32: round to nearest even; NaN -> canonical 0x7fff. */
static inline uint16_t bf16_rn(float f) {
  uint32_t u = bits_from_f32(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fffu;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline void store_elem(int dtype, void* out, int64_t i, float v) {
  if (dtype == OR_F32) ((float*)out)[i] = v;
  else if (dtype == OR_F16) ((_Float16*)out)[i] = (_Float16)v; /* cvt.rn.f16.f32 */
  else ((uint16_t*)out)[i] = bf16_rn(v);
}

static inline int log2i(int bs) { int l = 0; while ((1 << l) < bs) ++l; return l; }

int or_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ---------------------------------------------------------- code choice */

/* _quantize_nf4 (kernels/quantize.py:91-95): how many thresholds s exceeds. */
uint8_t or_code_nf4(float s) {
  int q = 0;
  for (int j = 0; j < 15; ++j) q += (s > f32_from_bits(NF4_THRESHOLD_BITS[j]));
  return (uint8_t)q;
}

/* _quantize_8bit (kernels/quantize.py:102-125): binary search of the sorted
 * codebook, then the nearer neighbour by midpoint. Literal restatement. */
uint8_t or_code_8bit(const float* C, float x) {
  int pivot = 127, upper_pivot = 255, lower_pivot = 0;
  float lower = -1.0f, upper = 1.0f;
  float val = C[pivot];
  for (int i = 64; i > 0; i >>= 1) {
    if (x > val) {
      lower_pivot = pivot; lower = val; pivot += i;
    } else {
      upper_pivot = pivot; upper = val; pivot -= i;
    }
    val = C[pivot];
  }
  if (upper_pivot == 255) upper = C[255];
  if (lower_pivot == 0) lower = C[0];
  if (x > val) return (uint8_t)((x > (upper + val) * 0.5f) ? upper_pivot : pivot);
  return (uint8_t)((x < (lower + val) * 0.5f) ? lower_pivot : pivot);
}

/* The same choice restated as a count of 255 strict thresholds, valid for a
 * strictly increasing finite codebook (the form the CUDA kernel evaluates).
 * Boundary j separates codes j and j+1; mid_j = fl(fl(C[j]+C[j+1]) * 0.5).
 * Even j is the "upper" test of leaf j (x > mid_j). Odd j is the "lower" test
 * of leaf j+1 (x >= mid_j, reached only when x > C[j]); as a strict test
 * that is x > pred(mid_j) when mid_j > C[j], else x > C[j]. Returns 1 when the
 * codebook qualifies, 0 otherwise (then only or_code_8bit applies). */
int or_q8_thresholds(const float* C, float* T) {
  for (int j = 0; j < 256; ++j)
    if (!isfinite(C[j])) return 0;
  for (int j = 0; j < 255; ++j)
    if (!(C[j] < C[j + 1])) return 0;
  for (int j = 0; j < 255; ++j) {
    float mid = (C[j] + C[j + 1]) * 0.5f;
    if (!(j & 1)) T[j] = mid;
    else T[j] = (mid > C[j]) ? nextafterf(mid, -INFINITY) : C[j];
  }
  return 1;
}

uint8_t or_code_8bit_count(const float* T, float x) {
  int c = 0;
  for (int j = 0; j < 255; ++j) c += (x > T[j]);
  return (uint8_t)c;
}

/* ------------------------------------------------------------- quantize */

/* Per-block absmax, kernels/quantize.py:153-164: m starts at -FLT_MAX and
 * folds max.ftz(m, abs.ftz(x)) over the block; the partial last block is read
 * zero-padded (kernels/quantize.py:221-225). */
static float block_absmax(int dtype, const void* x, int64_t n, int64_t b, int bs) {
  float m = -FLT_MAX;
  int64_t e0 = b * (int64_t)bs;
  for (int64_t i = 0; i < bs; ++i) {
    int64_t e = e0 + i;
    float v = (e < n) ? load_elem(dtype, x, e) : 0.0f;
    m = max_ftz(m, abs_ftz(v));
  }
  return m;
}

void or_absmax(int dtype, const void* x, int64_t n, int bs, float* absmax) {
  int64_t nb = (n + bs - 1) / bs;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) absmax[b] = block_absmax(dtype, x, n, b, bs);
}

/* Correctly rounded stand-in for rcp.approx.ftz.f32 (special values as the
 * PTX ISA defines them: 1/0 = +inf, 1/inf = 0; subnormal result -> 0). */
static inline float rcp_ieee_ftz(float m) { return ftz(1.0f / ftz(m)); }

void or_rcp_ieee_ftz(const float* m, float* r, int64_t nb) {
  for (int64_t b = 0; b < nb; ++b) r[b] = rcp_ieee_ftz(m[b]);
}

/* Reciprocal candidates when the device's value is not supplied. */
static int rcp_candidates(float m, float* c) {
  float r = rcp_ieee_ftz(m);
  if (isinf(r) || r == 0.0f || isnan(r)) { c[0] = r; return 1; }
  float lo = r, hi = r;
  int k = 0;
  c[k++] = r;
  for (int i = 0; i < 2; ++i) {
    lo = nextafterf(lo, -INFINITY);
    hi = nextafterf(hi, INFINITY);
    c[k++] = ftz(lo);
    c[k++] = ftz(hi);
  }
  return k;
}

/* quantize_nf4 (kernels/quantize.py:238-248 -> _quant_kernel :128-193 with
 * NF4=True): codes packed two per byte, high nibble first (:185-188); the
 * last byte of an odd n holds code(0 * r) in its low nibble (zero padding). */
void or_quantize_nf4(int dtype, const void* x, int64_t n, int bs, const float* rcp,
                     uint8_t* q, float* absmax, uint8_t* amb) {
  int64_t nb = (n + bs - 1) / bs;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    float m = block_absmax(dtype, x, n, b, bs);
    absmax[b] = m;
    float cand[5];
    int nc;
    if (rcp) { cand[0] = rcp[b]; nc = 1; }
    else nc = rcp_candidates(m, cand);
    int64_t e0 = b * (int64_t)bs, e1 = e0 + bs;
    if (e1 > n) e1 = n + (n & 1); /* the padding element of an odd n */
    for (int64_t e = e0; e < e1; ++e) {
      float v = (e < n) ? load_elem(dtype, x, e) : 0.0f;
      uint8_t c = or_code_nf4(mul_ftz(v, cand[0]));
      uint8_t a = 0;
      for (int k = 1; k < nc; ++k) a |= (or_code_nf4(mul_ftz(v, cand[k])) != c);
      if (amb && e < n) amb[e] = a;
      if (amb && e >= n && (e & 1) && a) amb[e - 1] = 1; /* padding nibble shares the byte */
      int64_t byte = e >> 1;
      if (e & 1) q[byte] = (uint8_t)((q[byte] & 0xF0u) | c);
      else q[byte] = (uint8_t)(c << 4);
    }
  }
}

/* quantize_blockwise (kernels/quantize.py:251-262 -> _quant_kernel NF4=False).
 * offset (nullable): elements are fl32(x - *offset) first (array.py:200-201). */
void or_quantize_8bit(int dtype, const void* x, int64_t n, int bs, const float* code,
                      const float* offset, const float* rcp, uint8_t* q, float* absmax,
                      uint8_t* amb) {
  int64_t nb = (n + bs - 1) / bs;
  float off = offset ? *offset : 0.0f;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    int64_t e0 = b * (int64_t)bs, e1 = e0 + bs < n ? e0 + bs : n;
    float m = -FLT_MAX;
    for (int64_t e = e0; e < e0 + bs; ++e) {
      float v = (e < n) ? load_elem(dtype, x, e) : 0.0f;
      if (offset && e < n) v = v - off;
      m = max_ftz(m, abs_ftz(v));
    }
    absmax[b] = m;
    float cand[5];
    int nc;
    if (rcp) { cand[0] = rcp[b]; nc = 1; }
    else nc = rcp_candidates(m, cand);
    for (int64_t e = e0; e < e1; ++e) {
      float v = load_elem(dtype, x, e);
      if (offset) v = v - off;
      uint8_t c = or_code_8bit(code, mul_ftz(v, cand[0]));
      uint8_t a = 0;
      for (int k = 1; k < nc; ++k) a |= (or_code_8bit(code, mul_ftz(v, cand[k])) != c);
      if (amb) amb[e] = a;
      q[e] = c;
    }
  }
}

/* ----------------------------------------------------------- dequantize */

/* _dequant_kernel (kernels/dequantize.py:39-69):
 *   out[i] = T(mul.ftz(table[q_i], absmax[i >> log2 bs]))
 * NF4: element 2j is the high nibble of byte j (:59-62). 8-bit: one byte per
 * element (:64-68). offset (nullable, 8-bit f32 only): + *offset afterwards,
 * the XLA add of a nested absmax (array.py:107-108). */
void or_dequantize(int nf4, int dtype, const uint8_t* q, const float* absmax,
                   const float* code, int64_t n, int bs, const float* offset, void* out) {
  int l2 = log2i(bs);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float a = absmax[i >> l2];
    float t;
    if (nf4) {
      uint8_t byte = q[i >> 1];
      t = NF4_TABLE[(i & 1) ? (byte & 15) : (byte >> 4)];
    } else {
      t = code[q[i]];
    }
    float v = mul_ftz(t, a);
    if (offset) v = v + *offset;
    store_elem(dtype, out, i, v);
  }
}

/* The nested absmax of a double-quantized array, as QuantizedArray.dequantize
 * decodes it (array.py:95-97 -> 8-bit dequantize at bs2, then + offset at
 * :107-108): a_b = fl32(mul.ftz(code2[aq_b], absmax2[(block0 + b) >> log2 bs2]) + offset). */
void or_nested_absmax(const uint8_t* aq, const float* absmax2, const float* code2,
                      float offset, int64_t nb, int bs2, int64_t block0, float* out) {
  int l2 = log2i(bs2);
  for (int64_t b = 0; b < nb; ++b)
    out[b] = mul_ftz(code2[aq[b]], absmax2[(block0 + b) >> l2]) + offset;
}

/* offset = mean(absmax): double accumulation, one rounding to float32. */
void or_mean(const float* a, int64_t n, float* out) {
  double s = 0.0;
  for (int64_t i = 0; i < n; ++i) s += a[i];
  *out = (float)(s / (double)n);
}

/* ----------------------------------------------------------------- GEMV */

/* Exact-as-possible product for the tolerance check: y[m][j] = sum_k x[m,k] *
 * w[j,k] in double, w = the float32 dequantized weight mul.ftz(table[q], a).
 * yabs[m][j] = sum_k |x[m,k] * w[j,k]| (scales the rounding bound). */
void or_gemv_f64(int dtype, const void* x, int m, int k, const uint8_t* w, int64_t n_rows,
                 int bs, const float* absmax, double* y, double* yabs) {
  int l2 = log2i(bs);
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n_rows; ++j) {
    for (int mi = 0; mi < m; ++mi) {
      double s = 0.0, sa = 0.0;
      for (int kk = 0; kk < k; ++kk) {
        int64_t e = j * (int64_t)k + kk;
        uint8_t byte = w[e >> 1];
        float t = NF4_TABLE[(e & 1) ? (byte & 15) : (byte >> 4)];
        double p = (double)load_elem(dtype, x, (int64_t)mi * k + kk) *
                   (double)mul_ftz(t, absmax[e >> l2]);
        s += p;
        sa += fabs(p);
      }
      y[(int64_t)mi * n_rows + j] = s;
      if (yabs) yabs[(int64_t)mi * n_rows + j] = sa;
    }
  }
}

/* The reference GEMV's own numerics (kernels/gemv.py:97-123): per 32-element
 * chunk t = sum table[q] * x in float32, acc += a * t, one rounding to the
 * output dtype. Used as the timed CPU baseline. */
void or_gemv_ref(int dtype, const void* x, int m, int k, const uint8_t* w, int64_t n_rows,
                 int bs, const float* absmax, void* y) {
  int l2 = log2i(bs);
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n_rows; ++j) {
    for (int mi = 0; mi < m; ++mi) {
      float acc = 0.0f;
      for (int c = 0; c < k; c += 32) {
        float t = 0.0f;
        int64_t e0 = j * (int64_t)k + c;
        for (int i = 0; i < 32; ++i) {
          int64_t e = e0 + i;
          uint8_t byte = w[e >> 1];
          float tv = NF4_TABLE[(e & 1) ? (byte & 15) : (byte >> 4)];
          t = t + tv * load_elem(dtype, x, (int64_t)mi * k + c + i);
        }
        acc = acc + absmax[e0 >> l2] * t;
      }
      store_elem(dtype, y, (int64_t)mi * n_rows + j, acc);
    }
  }
}

/* ----------------------------------------------- kernel-algorithm checks */

/* The NF4 quantize kernel replaces the 15-compare count by a bucket lookup:
 *   u = fma(max(s, -1), 16, 2^23 + 16)     (one rounding to an integer)
 *   i = bits(u) & 63                        (0..32 for |s| <= 1 + 2^-20)
 *   code = base[i] + (s > thr[i])
 * max() sends NaN to bucket 0 (code 0, as the count gives); the mask only
 * bounds the table index. The 64-entry tables are built from the thresholds'
 * own buckets (at most one threshold per bucket). or_check_nf4_buckets walks
 * every float32 s in [-1.01, 1.01] plus NaN and -inf and counts disagreements
 * with or_code_nf4. */
static inline int nf4_bucket(float s) {
  return (int)(bits_from_f32(fmaf(fmaxf(s, -1.0f), 16.0f, 8388624.0f)) & 63u);
}

int or_nf4_bucket_tables(float* thr, int32_t* base) {
  for (int i = 0; i < 64; ++i) {
    if (i <= 32) {
      int b = 0;
      thr[i] = INFINITY;
      for (int j = 0; j < 15; ++j) {
        float t = f32_from_bits(NF4_THRESHOLD_BITS[j]);
        int bt = nf4_bucket(t);
        if (bt < i) ++b;
        if (bt == i) {
          if (!isinf(thr[i])) return -1; /* two thresholds share a bucket */
          thr[i] = t;
        }
      }
      base[i] = b;
    } else {
      thr[i] = INFINITY;
      base[i] = 15; /* 33..63: above 1 + 1/32, unreachable for scaled values */
    }
  }
  return 0;
}

int64_t or_check_nf4_buckets(int64_t stride) {
  float thr[64];
  int32_t base[64];
  if (or_nf4_bucket_tables(thr, base) != 0) return -1;
  const uint32_t lo_pos = 0u, hi_pos = bits_from_f32(1.01f);
  int64_t bad = 0;
  if (stride < 1) stride = 1;
#pragma omp parallel for schedule(static) reduction(+ : bad)
  for (int64_t u = lo_pos; u <= (int64_t)hi_pos; u += stride) {
    for (int sgn = 0; sgn < 2; ++sgn) {
      float s = f32_from_bits((uint32_t)u | (sgn ? 0x80000000u : 0u));
      int i = nf4_bucket(s);
      int c = base[i] + (s > thr[i]);
      bad += (c != or_code_nf4(s));
    }
  }
  const float sp[4] = {NAN, -NAN, INFINITY, -INFINITY};
  for (int k = 0; k < 4; ++k) { /* NaN codes 0; +inf never reaches the kernel */
    if (sp[k] == INFINITY) continue;
    int i = nf4_bucket(sp[k]);
    bad += ((base[i] + (sp[k] > thr[i])) != or_code_nf4(sp[k]));
  }
  return bad;
}

/* The 8-bit kernel's code choice (csrc/bnbq_quant.cu, build_q8_tables and
 * code8_table), restated. Buckets by sign and magnitude key |bits| >> shift;
 * key 0 (below the smallest table threshold) and the key of 2.0 and above are
 * clamp buckets; NaN counts as -2. The largest mantissa-bit count mb = 23 -
 * shift whose keys fit Q8_KEYS per sign is used, first with all 255
 * thresholds, then with the smallest-magnitude one left out and compared
 * directly; it applies when every table threshold has a bucket of its own
 * that is not a clamp bucket. Entry E = base * 2^24 + (positive bucket:
 * 2^24 - 1 - low(T); negative: 2^24 + low(T) - 1), and code = (E + low(s)) >>
 * 24 for positive s, (E - low(s)) >> 24 for negative s. */
#define Q8_KEYS 4096

typedef struct {
  int shift, kmin, nkeys, ex;
  float t_ex;
} q8map;

static uint32_t q8_fine_index(const q8map* m, float s, uint32_t* low, uint32_t* sg) {
  uint32_t u = bits_from_f32(fmaxf(s, -2.0f)); /* NaN -> -2 */
  *sg = u >> 31;
  *low = u & ((1u << m->shift) - 1u);
  int32_t k = (int32_t)((u & 0x7fffffffu) >> m->shift) - m->kmin;
  k = k < 0 ? 0 : (k > m->nkeys - 1 ? m->nkeys - 1 : k);
  return *sg * (uint32_t)m->nkeys + (uint32_t)k;
}

static int q8_ord(int idx, int nkeys) { return idx >= nkeys ? nkeys - 1 - (idx - nkeys) : nkeys + idx; }

/* Builds the table from the 255 thresholds; returns mb, or -1 when the
 * formulation does not apply (the kernel then runs the literal search). */
int or_q8_fine_tables(const float* T, int32_t* map_out, uint32_t* tab, float* t_ex) {
  int jx = 0;
  for (int j = 1; j < 255; ++j)
    if ((bits_from_f32(T[j]) & 0x7fffffffu) < (bits_from_f32(T[jx]) & 0x7fffffffu)) jx = j;
  for (int ex = 0; ex < 2; ++ex) {
    for (int mb = 8; mb >= 1; --mb) {
      int shift = 23 - mb, kmin = 0x7fffffff;
      for (int j = 0; j < 255; ++j) {
        if (ex && j == jx) continue;
        int k = (int)((bits_from_f32(T[j]) & 0x7fffffffu) >> shift);
        kmin = k < kmin ? k : kmin;
      }
      kmin -= 1;
      int nkeys = (int)(0x40000000u >> shift) - kmin + 1;
      if (kmin < 0 || nkeys > Q8_KEYS) continue;
      q8map m = {shift, kmin, nkeys, ex, T[jx]};
      int ordc[255];
      uint32_t lowc[255];
      int nin = 0, ok = 1;
      for (int j = 0; j < 255 && ok; ++j) {
        if (ex && j == jx) continue;
        uint32_t low, sg;
        int idx = (int)q8_fine_index(&m, T[j], &low, &sg);
        int k = idx >= nkeys ? idx - nkeys : idx;
        if (k == 0 || k == nkeys - 1) ok = 0;
        ordc[nin] = q8_ord(idx, nkeys);
        lowc[nin] = low;
        if (nin > 0 && ordc[nin] <= ordc[nin - 1]) ok = 0;
        ++nin;
      }
      if (!ok) continue;
      uint32_t mask = (1u << shift) - 1u;
      for (int b = 0; b < 2 * nkeys; ++b) {
        int o = q8_ord(b, nkeys), lo = 0;
        while (lo < nin && ordc[lo] < o) ++lo;
        int neg = b >= nkeys;
        uint32_t lt = neg ? 0u : mask;
        if (lo < nin && ordc[lo] == o) lt = lowc[lo];
        tab[b] = (uint32_t)lo * (1u << 24) + (neg ? (1u << 24) + lt - 1u : (1u << 24) - 1u - lt);
      }
      map_out[0] = shift;
      map_out[1] = kmin;
      map_out[2] = nkeys;
      map_out[3] = ex;
      *t_ex = T[jx];
      return mb;
    }
  }
  return -1;
}

static uint8_t q8_fine_code(const q8map* m, const uint32_t* tab, float s) {
  uint32_t low, sg;
  uint32_t e = tab[q8_fine_index(m, s, &low, &sg)];
  uint32_t c = (sg ? e - low : e + low) >> 24;
  if (m->ex && s > m->t_ex) c += 1;
  return (uint8_t)c;
}

/* Walks float32 values in [-1.01, 1.01] at the given bit stride (plus NaN and
 * infinities) comparing the table formulation with the literal search.
 * Returns the mismatches (-1: the formulation does not apply), mb in *mb_out. */
int64_t or_check_q8_buckets(const float* C, int64_t stride, int* mb_out) {
  float T[255];
  int32_t mp[4];
  static uint32_t tab[2 * Q8_KEYS];
  if (!or_q8_thresholds(C, T)) return -1;
  float t_ex;
  int mb = or_q8_fine_tables(T, mp, tab, &t_ex);
  if (mb_out) *mb_out = mb;
  if (mb < 0) return -1;
  q8map m = {mp[0], mp[1], mp[2], mp[3], t_ex};
  const uint32_t hi_pos = bits_from_f32(1.01f);
  int64_t bad = 0;
  if (stride < 1) stride = 1;
#pragma omp parallel for schedule(static) reduction(+ : bad)
  for (int64_t u = 0; u <= (int64_t)hi_pos; u += stride) {
    for (int sgn = 0; sgn < 2; ++sgn) {
      float s = f32_from_bits((uint32_t)u | (sgn ? 0x80000000u : 0u));
      bad += (q8_fine_code(&m, tab, s) != or_code_8bit(C, s));
    }
  }
  /* every threshold and its neighbours within 3 ulp, both directions */
  for (int j = 0; j < 255; ++j) {
    float up = T[j], dn = T[j];
    for (int k = 0; k < 4; ++k) {
      bad += (q8_fine_code(&m, tab, up) != or_code_8bit(C, up));
      bad += (q8_fine_code(&m, tab, dn) != or_code_8bit(C, dn));
      up = nextafterf(up, INFINITY);
      dn = nextafterf(dn, -INFINITY);
    }
  }
  const float sp[6] = {NAN, -NAN, INFINITY, -INFINITY, 0.0f, -0.0f};
  for (int k = 0; k < 6; ++k) bad += (q8_fine_code(&m, tab, sp[k]) != or_code_8bit(C, sp[k]));
  return bad;
}

/* ------------------------------------------------- array forms (ctypes) */

void or_codes_nf4(const float* s, int64_t n, uint8_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = or_code_nf4(s[i]);
}

void or_codes_8bit(const float* C, const float* s, int64_t n, uint8_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = or_code_8bit(C, s[i]);
}

void or_codes_8bit_count(const float* T, const float* s, int64_t n, uint8_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = or_code_8bit_count(T, s[i]);
}

void or_mul_ftz(const float* a, const float* b, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = mul_ftz(a[i], b[i]);
}
