// Exhaustive check of the dithered encoder's delta division: Markstein's correction with the
// reciprocal pair (y_hi = RN(1/b), y_lo = RN(RN(1 - b*y_hi) * y_hi)) gives RN(a / b) for every
// finite float a >= 1e-8 (the encoder's floor on the absmax) and b = half = 1.5, 7.5, 127.5
// (2, 4 and 8 bits).  Exit status 1 if any quotient differs from IEEE division.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
static float bf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
int main(void) {
  const float halves[3] = {1.5f, 7.5f, 127.5f};
  uint64_t bad_total = 0;
  for (int k = 0; k < 3; ++k) {
    const float b = halves[k];
    const float yhi = 1.0f / b;
    const float e = fmaf(-b, yhi, 1.0f);
    const float ylo = e * yhi;
    uint64_t bad = 0, n = 0;
    for (uint32_t u = 0x322BCC77u; u < 0x7F800000u; ++u) {  // 1e-8 .. FLT_MAX
      const float a = bf(u);
      const float q0 = fmaf(a, yhi, a * ylo);
      const float r = fmaf(-q0, b, a);
      const float q1 = fmaf(r, yhi, q0);
      const float want = a / b;
      if (q1 != want) { if (bad < 5) printf("half %g a %a got %a want %a\n", b, a, q1, want); ++bad; }
      ++n;
    }
    printf("half %g: %llu of %llu wrong\n", b, (unsigned long long)bad, (unsigned long long)n);
    bad_total += bad;
  }
  return bad_total ? 1 : 0;
}
