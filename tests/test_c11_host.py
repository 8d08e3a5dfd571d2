"""The C-ABI as a C11 host sees it: a program that includes
include/gemma3_cuda.h compiled with gcc -std=c11 -pedantic -Werror (the
reference builds with -std=c11, gemma3.c Makefile), linked against
libgemma3_cuda.so, and run without a GPU.  Only host-side paths run: the
config defaults, the RoPE table helper, and the argument checks of entry
points (a NULL context, an unsupported configuration) that must fail with
GEMMA3_CUDA_ERR_INVALID_ARG before touching a device."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "gemma3.c_b200")

PROGRAM = r"""
#include <math.h>
#include <stdio.h>
#include <string.h>
#include "gemma3_cuda.h"

static int fails = 0;
#define CHECK(c) do { if (!(c)) { printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #c); ++fails; } } while (0)

int main(void) {
    gemma3_cuda_config cfg;
    gemma3_cuda_config_default(&cfg);
    CHECK(cfg.num_layers == 34 && cfg.num_heads == 8 && cfg.num_kv_heads == 4);
    CHECK(cfg.head_dim == 256 && cfg.sliding_window == 1024);
    CHECK(cfg.kv_ranks == 1 && cfg.kv_rank == 0);

    /* the reference's table formula: freq = 1/theta^(2i/d), angle = pos*freq */
    static float tab[4 * 128 * 2];
    gemma3_cuda_rope_precompute(tab, 4, 256, 10000.0f);
    CHECK(tab[0] == 1.0f && tab[1] == 0.0f);
    CHECK(fabsf(tab[(3 * 128 + 1) * 2 + 1] - sinf(3.0f / powf(10000.0f, 2.0f / 256.0f))) < 1e-6f);

    /* unsupported geometry: rejected before any device work */
    gemma3_cuda_config bad = cfg;
    bad.head_dim = 128;
    CHECK(gemma3_cuda_init(&bad) == NULL);
    CHECK(strlen(gemma3_cuda_last_error()) > 0);
    CHECK(gemma3_cuda_init(NULL) == NULL);

    /* NULL contexts */
    CHECK(gemma3_cuda_synchronize(NULL) == GEMMA3_CUDA_ERR_INVALID_ARG);
    CHECK(gemma3_cuda_peer_init(NULL) == GEMMA3_CUDA_ERR_INVALID_ARG);
    CHECK(gemma3_cuda_set_exchange(NULL, GEMMA3_CUDA_XCHG_PEER) == GEMMA3_CUDA_ERR_INVALID_ARG);
    CHECK(gemma3_cuda_reset(NULL) == GEMMA3_CUDA_ERR_INVALID_ARG);
    CHECK(gemma3_cuda_stream(NULL) == NULL);
    gemma3_cuda_free(NULL);

    /* the no-allocation decode rejects a batch beyond its static scratch */
    {   /* rejected by its size check, before any pointer is used */
        static float dummy[16];
        static int nrows[65];
        CHECK(gemma3_cuda_gqa_decode_noalloc(dummy, dummy, GEMMA3_CUDA_KV_BF16, 1024, 65, nrows, dummy, NULL) ==
              GEMMA3_CUDA_ERR_INVALID_ARG);
        CHECK(strstr(gemma3_cuda_last_error(), "B=65") != NULL);
    }
    printf("%s\n", fails ? "FAILED" : "OK");
    return fails != 0;
}
"""


def test_c11_host_program(tmp_path):
    lib = os.path.join(LIBDIR, "libgemma3_cuda.so")
    if not os.path.exists(lib):
        pytest.fail("libgemma3_cuda.so not built: run `make -C gemma3.c_b200 cuda`")
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    cc = subprocess.run(["gcc", "-std=c11", "-pedantic", "-Wall", "-Wextra", "-Werror",
                         "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                         "-L", LIBDIR, "-lgemma3_cuda", "-lm", f"-Wl,-rpath,{LIBDIR}"],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    # no GPU is needed for these paths; hide any that exists so none is touched
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    run = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=120)
    assert run.returncode == 0 and run.stdout.strip().endswith("OK"), run.stdout + run.stderr
