#include <stdio.h>
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static uint32_t byte_perm(uint32_t x, uint32_t y, uint32_t s) {
  uint64_t v = ((uint64_t)y << 32) | x; uint32_t r = 0;
  for (int i = 0; i < 4; ++i) { int sel = (s >> (4 * i)) & 7; r |= (uint32_t)((v >> (8 * sel)) & 0xFF) << (8 * i); }
  return r;
}
static uint32_t biased24(float x, float sc) { return f2u(fmaf(x, sc, 12582912.0f)) - (0x4B400000u - 0x808080u); }
static int old_digits(float x, float sc, int d[3]) {
  int a = (int)nearbyintf(x * sc);
  d[0] = ((a + 128) & 255) - 128; int r1 = (a - d[0]) >> 8;
  d[1] = ((r1 + 128) & 255) - 128; d[2] = (r1 - d[1]) >> 8; return a;
}
int main(void) {
  srand(1); long bad = 0, n = 0;
  for (int it = 0; it < 2000000; ++it) {
    float v[4]; int e = (rand() % 60) - 30; float sc = ldexpf(1.f, 22 - e);
    for (int j = 0; j < 4; ++j) { float r = ((float)rand() / RAND_MAX * 2.f - 1.f); v[j] = ldexpf(r, e); if (rand() % 50 == 0) v[j] = ldexpf(((rand()%2)?1:-1)*(0.5f + (rand()%1000)/2000.f), e); }
    // halfway cases
    if (it % 97 == 0) v[0] = ldexpf(2.5f, -22 + e) ;
    uint32_t u[4]; for (int j = 0; j < 4; ++j) u[j] = biased24(v[j], sc);
    uint32_t t01 = byte_perm(u[0], u[1], 0x5140), t23 = byte_perm(u[2], u[3], 0x5140);
    uint32_t s01 = byte_perm(u[0], u[1], 0x0062), s23 = byte_perm(u[2], u[3], 0x0062);
    uint32_t w[3] = {byte_perm(t01, t23, 0x5410) ^ 0x80808080u, byte_perm(t01, t23, 0x7632) ^ 0x80808080u,
                     byte_perm(s01, s23, 0x5410) ^ 0x80808080u};
    int sum = (int)((u[0] + u[1]) + (u[2] + u[3]) - 4u * 0x808080u), osum = 0;
    for (int j = 0; j < 4; ++j) {
      int d[3]; osum += old_digits(v[j], sc, d);
      for (int q = 0; q < 3; ++q) { int nd = (int8_t)((w[q] >> (8 * j)) & 0xFF); if (nd != d[q]) ++bad; }
    }
    if (sum != osum) ++bad;
    ++n;
  }
  printf("checked %ld float4, mismatches %ld\n", n, bad);
  return bad != 0;
}
