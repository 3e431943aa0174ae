"""The C ABI library on CPU: it loads, exports every function include/rt_b200.h declares, keeps
struct rt's layout, and computes sizes without a GPU. No product runs here."""
from __future__ import annotations

import ctypes as C
import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "rt_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:RTB_API\s+)?(?:const\s+)?[a-z_0-9]+\s*\**\s*([a-z_0-9]+)\s*\(", text, flags=re.M)
    return [n for n in names if n not in ("if", "return")]


def test_header_declares_the_reference_products():
    names = set(declared_functions())
    # src/card/rt.h:39, 62-72, 85
    for f in ("rt_init", "rt_gemv", "rt_gemv_q", "rt_gemv_open", "rt_gemv_go", "rt_gemm", "rt_gemm_q", "rt_q8_row"):
        assert f in names, f


def test_library_exports_every_declared_symbol(rtb):
    lib = rtb.load()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(rtb.EXPORTS)


def test_struct_rt_layout(rtb):
    # src/card/rt.h:19-26 on x86-64: four pointers then two ints
    assert C.sizeof(rtb.StructRt) == 40
    assert rtb.StructRt.threads.offset == 32 and rtb.StructRt.last.offset == 36


def test_split_sizes(rtb, oracle):
    for rows, cols in [(1, 32), (7, 96), (4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]:
        assert rtb.gemv_s_bytes(rows, cols) == oracle.port().q8o_split_bytes(rows, cols)
    assert rtb.gemv_s_bytes(4096, 4096) == 4096 * 4096 * 34 // 32
    assert rtb.gemv_s_bytes(4, 33) == -1


def test_calls_without_init_record_an_error(rtb):
    lib = rtb.load()
    R = rtb.StructRt()
    lib.rt_gemv(C.byref(R), None, 16, 32, None, None)  # R.chain NULL: no device work attempted
    code, msg = rtb.last_error(None)
    assert code == 5 and "rt_init" in msg
    assert rtb.last_error(None)[0] == 0  # reading clears
    assert lib.rt_b200_wait_probe(C.byref(R)) == 5  # the failure self-test needs rt_init too
    assert rtb.last_error(None)[0] == 5


# A C translation unit shaped like the engine's generated model code (a struct rt on the stack,
# products on frame addresses, a queued round closed by rt_gemv_go): it must compile as C against
# include/rt_b200.h and link against the library unchanged. Run without rt_init, every product
# records RTB_ENOTINIT and touches no device.
GENERATED_STYLE_C = r"""
#include <stdio.h>
#include "rt_b200.h"

static float frame[4096 + 64] __attribute__((aligned(64)));

int main(void)
{
    struct rt R = {0};
    R.frame = (char *)frame;
    const void *W = (const void *)0x1000;
    float *X = frame, *V = frame + 4096;
    int codes[8], k = 0;
    rt_gemv(&R, W, 16, 4096, X, V);
    codes[k++] = rt_b200_last_error(NULL, NULL, 0);
    rt_gemv_open(&R);
    codes[k++] = rt_b200_last_error(NULL, NULL, 0);
    rt_gemv_q(&R, W, 16, 4096, X, V);
    codes[k++] = rt_b200_last_error(NULL, NULL, 0);
    rt_gemm_q(&R, W, 16, 256, X, 16, V);
    codes[k++] = rt_b200_last_error(NULL, NULL, 0);
    rt_gemv_go(&R);
    codes[k++] = rt_b200_last_error(NULL, NULL, 0);
    rt_gemm(&R, W, 16, 256, X, 2, V);
    codes[k++] = rt_b200_last_error(NULL, NULL, 0);
    for (int i = 0; i < k; i++)
        printf("%d ", codes[i]);
    printf("| %ld %ld\n", gemv_s_bytes(4096, 4096), (long)sizeof(struct rt));
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_generated_style_c_code_compiles_and_links(rtb, tmp_path):
    rtb.load()  # the library is built
    src = tmp_path / "model_card.c"
    src.write_text(GENERATED_STYLE_C)
    exe = tmp_path / "model_card"
    pkg = os.path.dirname(rtb.LIB_PATH)
    cc = subprocess.run(["gcc", "-std=gnu11", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                         str(src), "-o", str(exe), f"-L{pkg}", "-l:librt_b200.so", f"-Wl,-rpath,{pkg}"],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    codes, sizes = run.stdout.strip().split("|")
    assert codes.split() == ["5"] * 6  # RTB_ENOTINIT for every product: nothing reached a device
    assert sizes.split() == [str(4096 * 4096 * 34 // 32), "40"]


# The engine's load site (src/card/engine.c:295-316 of the reference): scratch sized by
# gemv_i_bytes, one struct gemv_repack_job per matrix, run as a team body on every thread. It must
# compile and link against the library under the reference's names. Run on the host: threads other
# than 0 return at once, and thread 0 refuses an in-place repack whose rows would change length
# (cols % 256 != 0) before touching a device.
LOAD_SITE_C = r"""
#include <stdio.h>
#include <stdint.h>
#include "rt_b200.h"

static void team_run(void (*fn)(void *, int, int), void *arg, int n)
{
    for (int tid = n - 1; tid >= 0; tid--)  /* tid 0 is the caller's thread, as in the engine */
        fn(arg, tid, n);
}

int main(void)
{
    long max_cols = 12288;
    long scratch = gemv_i_bytes(16, max_cols) * 4;
    struct gemv_repack_job rj = {.w = (void *)0x1000, .rows = 64, .cols = 4128, .tmp = 0};
    gemv_i_repack_thread(&rj, 3, 4);
    int other = rt_b200_last_error(NULL, NULL, 0);
    team_run(gemv_i_repack_thread, &rj, 4);
    int refused = rt_b200_last_error(NULL, NULL, 0);
    gemv_i_repack((const uint8_t *)0, 64, 4096, (void *)0x1000);
    int null_arg = rt_b200_last_error(NULL, NULL, 0);
    printf("%ld %ld %d %d %d\n", scratch, gemv_i_bytes(4096, 4096), other, refused, null_arg);
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_engine_load_site_links_under_the_reference_names(rtb, tmp_path):
    rtb.load()
    src = tmp_path / "load_site.c"
    src.write_text(LOAD_SITE_C)
    exe = tmp_path / "load_site"
    pkg = os.path.dirname(rtb.LIB_PATH)
    cc = subprocess.run(["gcc", "-std=gnu11", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                         str(src), "-o", str(exe), f"-L{pkg}", "-l:librt_b200.so", f"-Wl,-rpath,{pkg}"],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    scratch, full, other, refused, null_arg = run.stdout.split()
    assert int(scratch) == 4 * 16 * 12288 * 34 // 32 and int(full) == 4096 * 4096 * 34 // 32
    assert (other, refused, null_arg) == ("0", "1", "1")  # RTB_EINVAL, before any device call
