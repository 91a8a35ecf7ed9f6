"""The C oracle (oracle/c/oracle.c) built with AddressSanitizer and UndefinedBehaviorSanitizer
around a small C driver: the router, dequant, RMSNorm and exp on random and special inputs
(NaN / Inf / subnormal f16 fields, a zero row, extreme exp arguments) run without a sanitizer
report. The kernels cannot be built for the host, so this is the host-side check of the code
they are compared against. CPU only."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

DRIVER = r'''
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
float b2o_expf(float x);
void b2o_q4k_dequant(const uint8_t *blk, int64_t nb, float *out);
void b2o_router(const float *x, int T, const uint16_t *wg, const float *bias, uint16_t *logits_out,
                float *probs_out, int32_t *ids, float *w_f32, uint16_t *w_bf16);
void b2o_rmsnorm(const float *x, int T, float eps, float *y);
static uint32_t s = 12345u;
static uint32_t rnd(void) { s = s * 1664525u + 1013904223u; return s >> 8; }
static float unif(void) { return (float)(rnd() & 0xFFFFFF) / 16777216.0f - 0.5f; }
int main(void) {
  enum { T = 3, H = 2048, E = 256, NB = 64 };
  float *x = malloc(sizeof(float) * T * H), *y = malloc(sizeof(float) * T * H);
  uint16_t *wg = malloc(sizeof(uint16_t) * E * H), *lg = malloc(sizeof(uint16_t) * T * E);
  float *pr = malloc(sizeof(float) * T * E), *wf = malloc(sizeof(float) * T * 8);
  int32_t *ids = malloc(sizeof(int32_t) * T * 8);
  uint16_t *wb = malloc(sizeof(uint16_t) * T * 8);
  for (int i = 0; i < T * H; ++i) x[i] = (i < H) ? 0.0f : unif() * 0.05f;  /* row 0: all zero */
  for (int i = 0; i < E * H; ++i) wg[i] = (uint16_t)(rnd() & 0x3FFF);    /* finite bf16 */
  b2o_router(x, T, wg, NULL, lg, pr, ids, wf, wb);
  for (int i = 0; i < T * 8; ++i) if (ids[i] < 0 || ids[i] >= E) return 2;
  b2o_rmsnorm(x + H, T - 1, 1e-6f, y);
  uint8_t *blk = malloc(144 * NB);
  float *out = malloc(sizeof(float) * 256 * NB);
  for (int i = 0; i < 144 * NB; ++i) blk[i] = (uint8_t)rnd();
  const uint16_t special[] = {0x7C00, 0xFC00, 0x7E00, 0x0001, 0x8000, 0x7BFF};  /* inf, -inf, nan, subnormal, -0, max */
  for (int b = 0; b < 6; ++b) { memcpy(blk + 144 * b, &special[b], 2); memcpy(blk + 144 * b + 2, &special[5 - b], 2); }
  b2o_q4k_dequant(blk, NB, out);
  const float xs[] = {0.0f, -0.0f, 1.0f, -1.0f, 88.7f, 89.0f, -103.9f, -104.0f, -1e30f, 1e30f, NAN, INFINITY, -INFINITY};
  float acc = 0.0f;
  for (unsigned i = 0; i < sizeof xs / sizeof xs[0]; ++i) acc += isnan(b2o_expf(xs[i])) ? 0.0f : 1.0f;
  printf("ok %d %g\n", ids[0], (double)acc);
  free(x); free(y); free(wg); free(lg); free(pr); free(wf); free(ids); free(wb); free(blk); free(out);
  return 0;
}
'''


def test_oracle_under_asan_ubsan(tmp_path):
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    drv = tmp_path / "drv.c"
    drv.write_text(DRIVER)
    exe = tmp_path / "drv"
    cmd = ["gcc", "-O1", "-g", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fno-builtin",
           "-fsanitize=address,undefined", "-fno-sanitize-recover=all", "-fno-omit-frame-pointer",
           str(drv), os.path.join(ROOT, "oracle", "c", "oracle.c"), "-lm", "-o", str(exe)]
    try:
        subprocess.run(cmd, check=True, capture_output=True, text=True)
    except subprocess.CalledProcessError as e:
        if "sanitize" in (e.stderr or "") and "cannot find" in (e.stderr or ""):
            pytest.skip("sanitizer runtime not installed")
        raise
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=env)
    if "LeakSanitizer has encountered a fatal error" in r.stderr:  # no ptrace here: leaks unchecked
        env["ASAN_OPTIONS"] = "detect_leaks=0:abort_on_error=0"
        r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and r.stdout.startswith("ok"), (r.returncode, r.stdout, r.stderr[-2000:])
    assert "runtime error" not in r.stderr and "ERROR: AddressSanitizer" not in r.stderr, r.stderr[-2000:]
