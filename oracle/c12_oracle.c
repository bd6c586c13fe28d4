/*
 * CPU oracle (C port) for the 12-bit lossless BF16 weight format and the small-M projection.
 *
 * TEST INFRASTRUCTURE ONLY: linked by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs as the checker and CPU baseline. The product path never loads this library.
 *
 * Restates the reference (NathenFernandes/muse-bf16-proj, submission.py = "S"):
 *   unit layout            S:82-87    (lane l = 4g+t, value v = 8q+4hf+2rh+d -> row 8rh+g, col 16t+4q+2hf+d)
 *   12-bit pack            S:104-125  (base = first argmax of 8-wide exponent windows, d = exp7-base, escapes)
 *   12-bit unpack          S:128-142
 *   projection semantics   S:2610-2617 (x @ W.T, FP32 accumulate, BF16 round-to-nearest-even)
 * with two generalisations that reduce to the reference exactly: per-16-row-tile bases (tile_base=1) and an
 * unbounded compressed-sparse escape list (entry = c<<17 | lane<<12 | v<<7 | xor7, offsets per unit).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define UNIT_BYTES 1536
static const int SIGN_POS[8] = {3, 19, 7, 23, 11, 27, 15, 31};

/* row / column of value v of lane l inside a 16x64 unit (S:84-86) */
static inline int unit_row(int lane, int v) { return ((v >> 1) & 1) * 8 + (lane >> 2); }
static inline int unit_col(int lane, int v) {
  return (lane & 3) * 16 + (v >> 3) * 4 + ((v >> 2) & 1) * 2 + (v & 1);
}

static int window_base(const int64_t* hist) {
  int best = 0;
  int64_t bestv = -1;
  for (int b = 0; b < 121; ++b) {
    int64_t s = 0;
    for (int i = 0; i < 8; ++i) s += hist[b + i];
    if (s > bestv) { bestv = s; best = b; }
  }
  return best;
}

int orc_version(void) { return 1; }

/* Pack W (BF16 bits, row-major [n, k]) into units [n/16][k/64][1536], bases [n/16] and a CSR escape list.
 * Returns the escape count, or -1 when it exceeds esc_cap (esc may be NULL with esc_cap 0 to count only),
 * or -2 for a bad shape. */
int64_t orc_pack_c12(const uint16_t* w, int n, int k, int tile_base, uint8_t* units, uint8_t* bases,
                     int32_t* esc_off, uint32_t* esc, int64_t esc_cap) {
  if (n <= 0 || k <= 0 || n % 16 || k % 64 || k / 64 >= (1 << 15)) return -2;
  const int R = n / 16, C = k / 64;
  int64_t* hist = (int64_t*)calloc((size_t)R * 128, sizeof(int64_t));
  for (int r = 0; r < R; ++r)
    for (size_t i = (size_t)r * 16 * k; i < (size_t)(r + 1) * 16 * k; ++i) hist[(size_t)r * 128 + ((w[i] >> 8) & 0x7F)]++;
  if (tile_base) {
    for (int r = 0; r < R; ++r) bases[r] = (uint8_t)window_base(hist + (size_t)r * 128);
  } else {
    int64_t tot[128] = {0};
    for (int r = 0; r < R; ++r)
      for (int e = 0; e < 128; ++e) tot[e] += hist[(size_t)r * 128 + e];
    int b = window_base(tot);
    for (int r = 0; r < R; ++r) bases[r] = (uint8_t)b;
  }
  free(hist);
  int64_t ne = 0;
  for (int r = 0; r < R; ++r) {
    const int base = bases[r];
    for (int c = 0; c < C; ++c) {
      uint8_t* u = units + ((size_t)r * C + c) * UNIT_BYTES;
      if (esc_off) esc_off[(size_t)r * C + c] = (int32_t)ne;
      for (int lane = 0; lane < 32; ++lane) {
        uint32_t code[4] = {0, 0, 0, 0};
        for (int v = 0; v < 32; ++v) {
          const uint16_t x = w[(size_t)(r * 16 + unit_row(lane, v)) * k + c * 64 + unit_col(lane, v)];
          const int eh = (x >> 8) & 0x7F, sg = x >> 15;
          int d = eh - base;
          if (d < 0 || d >= 8) {
            if (esc) {
              if (ne >= esc_cap) return -1;
              esc[ne] = ((uint32_t)c << 17) | ((uint32_t)lane << 12) | ((uint32_t)v << 7) | (uint32_t)(eh ^ base);
            }
            ++ne;
            d = 0;
          }
          u[(v >> 4) * 512 + lane * 16 + (v & 15)] = (uint8_t)(x & 0xFF);
          code[v >> 3] |= ((uint32_t)d << (4 * (v & 7))) | ((uint32_t)sg << SIGN_POS[v & 7]);
        }
        memcpy(u + 1024 + lane * 16, code, 16);
      }
    }
  }
  if (esc_off) esc_off[(size_t)R * C] = (int32_t)ne;
  return ne;
}

/* Decodes one unit into float weights wt[16][64] (row, col inside the unit). */
static void decode_unit_f32(const uint8_t* u, int base, const uint32_t* e0, const uint32_t* e1, float* wt) {
  uint16_t vals[32][32];
  for (int lane = 0; lane < 32; ++lane) {
    uint32_t code[4];
    memcpy(code, u + 1024 + lane * 16, 16);
    for (int v = 0; v < 32; ++v) {
      const uint32_t cw = code[v >> 3];
      const int i = v & 7;
      const uint32_t d = (cw >> (4 * i)) & 7, sg = (cw >> SIGN_POS[i]) & 1;
      vals[lane][v] = (uint16_t)((sg << 15) | ((base + d) << 8) | u[(v >> 4) * 512 + lane * 16 + (v & 15)]);
    }
  }
  for (const uint32_t* e = e0; e < e1; ++e) vals[(*e >> 12) & 31][(*e >> 7) & 31] ^= (uint16_t)((*e & 0x7F) << 8);
  for (int lane = 0; lane < 32; ++lane)
    for (int v = 0; v < 32; ++v) {
      uint32_t b = (uint32_t)vals[lane][v] << 16;
      float f;
      memcpy(&f, &b, 4);
      wt[unit_row(lane, v) * 64 + unit_col(lane, v)] = f;
    }
}

/* Exact inverse of orc_pack_c12: units + bases + escapes -> W (BF16 bits). */
int orc_unpack_c12(const uint8_t* units, const uint8_t* bases, const int32_t* esc_off, const uint32_t* esc, int n,
                   int k, uint16_t* w) {
  if (n % 16 || k % 64) return -2;
  const int R = n / 16, C = k / 64;
  for (int r = 0; r < R; ++r)
    for (int c = 0; c < C; ++c) {
      const uint8_t* u = units + ((size_t)r * C + c) * UNIT_BYTES;
      float wt[16 * 64];
      decode_unit_f32(u, bases[r], esc + esc_off[(size_t)r * C + c], esc + esc_off[(size_t)r * C + c + 1], wt);
      for (int i = 0; i < 16; ++i)
        for (int j = 0; j < 64; ++j) {
          uint32_t b;
          memcpy(&b, &wt[i * 64 + j], 4);
          w[(size_t)(r * 16 + i) * k + c * 64 + j] = (uint16_t)(b >> 16);
        }
    }
  return 0;
}

static inline float bf2f(uint16_t h) {
  uint32_t b = (uint32_t)h << 16;
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (isnan(f)) return (uint16_t)((u >> 16) | 0x40);
  return (uint16_t)((u + 0x7FFF + ((u >> 16) & 1)) >> 16);
}

/* out[m, n] = x[m, k] . W^T from the packed format: the projection of S:2610-2617 computed the way the GPU path
 * computes it (decode, FP32 accumulate per output). out_f32 and/or out_bf16 may be NULL.
 * Rows [row0, row0 + nrows) only (a bounded sample); threads <= 0 uses all. */
int orc_gemv_c12(const uint16_t* x, int m, const uint8_t* units, const uint8_t* bases, const int32_t* esc_off,
                 const uint32_t* esc, int n, int k, int row0, int nrows, float* out_f32, uint16_t* out_bf16,
                 int threads) {
  if (n % 16 || k % 64 || row0 % 16 || nrows % 16 || row0 + nrows > n) return -2;
  const int C = k / 64;
  float* xf = (float*)malloc(sizeof(float) * (size_t)m * k);
  for (size_t i = 0; i < (size_t)m * k; ++i) xf[i] = bf2f(x[i]);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(dynamic, 1)
  for (int r = row0 / 16; r < (row0 + nrows) / 16; ++r) {
    float acc[16 * 256];
    float wt[16 * 64];
    for (int mb = 0; mb < m; mb += 256) {
      const int mm = m - mb < 256 ? m - mb : 256;
      memset(acc, 0, sizeof(float) * 16 * (size_t)mm);
      for (int c = 0; c < C; ++c) {
        const size_t ui = (size_t)r * C + c;
        decode_unit_f32(units + ui * UNIT_BYTES, bases[r], esc + esc_off[ui], esc + esc_off[ui + 1], wt);
        for (int t = 0; t < mm; ++t) {
          const float* xr = xf + (size_t)(mb + t) * k + c * 64;
          for (int i = 0; i < 16; ++i) {
            float s = 0.f;
            for (int j = 0; j < 64; ++j) s += xr[j] * wt[i * 64 + j];
            acc[t * 16 + i] += s;
          }
        }
      }
      for (int t = 0; t < mm; ++t)
        for (int i = 0; i < 16; ++i) {
          const size_t o = (size_t)(mb + t) * n + r * 16 + i;
          if (out_f32) out_f32[o] = acc[t * 16 + i];
          if (out_bf16) out_bf16[o] = f2bf(acc[t * 16 + i]);
        }
    }
  }
  free(xf);
  return 0;
}

/* Dense reference: out[m, n] = x . W^T with BF16 inputs and FP64 accumulation (the FP64 check of S:297-317). */
int orc_linear_f64(const uint16_t* x, const uint16_t* w, int m, int n, int k, double* out, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(static)
  for (int j = 0; j < n; ++j)
    for (int t = 0; t < m; ++t) {
      double s = 0.0;
      for (int i = 0; i < k; ++i) s += (double)bf2f(x[(size_t)t * k + i]) * (double)bf2f(w[(size_t)j * k + i]);
      out[(size_t)t * n + j] = s;
    }
  return 0;
}

/* Router reference: out[m, n] = x_bf16 . W_f32^T in FP64 (S:2613-2617 semantics, exact weights). */
int orc_linear_xbf16_wf32_f64(const uint16_t* x, const float* w, int m, int n, int k, double* out, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(static)
  for (int j = 0; j < n; ++j)
    for (int t = 0; t < m; ++t) {
      double s = 0.0;
      for (int i = 0; i < k; ++i) s += (double)bf2f(x[(size_t)t * k + i]) * (double)w[(size_t)j * k + i];
      out[(size_t)t * n + j] = s;
    }
  return 0;
}
