"""CPU tests of the drop-in boundary: libw4a16.so loads and exports every symbol
include/w4a16.h declares, host-side validation follows the reference's check
order and messages (kernel.cu:219-249), and the torch binding's tensor checks."""
import ctypes
import os
import re

import pytest
import torch

from w4a16_opt import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "w4a16.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w4a16_[a-z_]+)\s*\(", text)))


def test_header_declares_exports_table():
    assert declared_functions() == sorted(capi.EXPORTS)


def test_library_loads_and_exports_every_symbol():
    lib = capi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.w4a16_abi_version() == 4


def test_library_has_no_torch_dependency():
    # The C ABI is usable from any host language: no libtorch/libc10 in its link map.
    import subprocess
    out = subprocess.run(["ldd", capi.library_path()], capture_output=True, text=True).stdout
    # library names only: the hex load addresses ldd prints are random and may contain "c10"
    names = [line.split()[0] for line in out.splitlines() if line.strip()]
    assert names and not any("torch" in n or "c10" in n for n in names), names


def test_status_strings():
    lib = capi.load()
    for code, name in capi.STATUS_NAMES.items():
        assert lib.w4a16_status_string(code).decode() == name


def _validate(M=2, N=64, K=512, groups=8, wp_words=None, variant=-1, wp=None, x=None, s=None):
    lib = capi.load()
    wp_words = N * K // 8 if wp_words is None else wp_words
    st = lib.w4a16_validate(wp, x, s, M, N, K, groups, wp_words, variant)
    return st, capi.last_error(lib)


@pytest.mark.parametrize("kw,status,msg", [
    (dict(variant=7), 2, "variant must be -1 (auto), 0 (decode) or 1..4"),
    (dict(variant=-2), 2, "variant"),
    (dict(M=0), 3, "M must be at least 1"),
    (dict(N=1 << 31, groups=8), 4, "dimensions must fit in int32"),
    (dict(K=32, groups=1), 5, "multiple of 64"),
    (dict(N=24), 6, "multiple of 16"),
    (dict(groups=3), 7, "divisible by the number of groups"),
    (dict(wp_words=5), 8, "Wp must hold N*K/8 words"),
    (dict(wp=0x1008), 9, "16-byte aligned"),
    (dict(groups=16), 10, "unsupported group size 32, supported: 64, 128"),
    (dict(groups=2), 10, "unsupported group size 256"),
    (dict(M=32, variant=0), 11, "decode kernel needs"),
    (dict(N=80, K=640, groups=10, variant=0), 11, "decode kernel needs"),
])
def test_validate_rejects(kw, status, msg):
    st, err = _validate(**kw)
    assert st == status, (st, err)
    assert msg in err


def test_validate_check_order():
    # variant is checked before the shapes, K before N, groups before the word count
    assert _validate(variant=9, M=0)[0] == 2
    assert _validate(K=32, N=24, groups=1)[0] == 5
    assert _validate(groups=3, wp_words=1)[0] == 7


@pytest.mark.parametrize("kw", [dict(), dict(variant=0), dict(variant=3, M=1000), dict(N=208, K=384, groups=3)])
def test_validate_accepts(kw):
    assert _validate(**kw)[0] == 0


def test_gemm_null_pointers_rejected():
    lib = capi.load()
    st = lib.w4a16_gemm(None, None, None, None, 2, 64, 512, 8, 64 * 512 // 8, -1, 0, None, 0, None)
    assert st == 1 and "non-null" in capi.last_error(lib)


def test_gemm_unknown_flags_rejected():
    lib = capi.load()
    p = ctypes.c_void_p(0x10000)
    st = lib.w4a16_gemm_ex(p, p, p, p, 2, 64, 512, 8, 64 * 512 // 8, -1, 0, 4, None, 0, None)
    assert st == 17 and "unknown flag bits 4" in capi.last_error(lib)


def test_gemm_bad_out_dtype_rejected():
    lib = capi.load()
    p = ctypes.c_void_p(0x10000)
    st = lib.w4a16_gemm(p, p, p, p, 2, 64, 512, 8, 64 * 512 // 8, -1, 5, None, 0, None)
    assert st == 12


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_query_route_without_gpu_reports_cuda_error():
    lib = capi.load()
    r = capi.Route()
    st = lib.w4a16_query_route(1, 4096, 4096, 32, -1, ctypes.byref(r))
    assert st in (13, 14)


# ---------------------------------------------------------------- torch binding tensor checks (CPU)

def test_binding_rejects_cpu_tensors():
    from w4a16_opt import w4a16_gemm
    Wp = torch.zeros(64 * 512 // 8, dtype=torch.int32)
    x = torch.zeros(2, 512, dtype=torch.half)
    s = torch.zeros(8, 64, dtype=torch.half)
    with pytest.raises(RuntimeError, match="CUDA"):
        w4a16_gemm(Wp, x, s)


def test_binding_exports():
    import w4a16_opt
    for name in ("w4a16_gemm", "w4a16_gemm_out", "w4a16_dequant", "query_route", "device_status"):
        assert callable(getattr(w4a16_opt, name))
    assert w4a16_opt.ABI_VERSION == 4


@pytest.mark.skipif(__import__("shutil").which("gcc") is None, reason="needs gcc")
def test_header_layout_matches_ctypes(tmp_path):
    """include/w4a16.h compiles as C99, and its struct layout and status codes are the ones
    the ctypes binding declares (what a cgo / JNI / N-API binding would also rely on)."""
    import subprocess
    fields = [name for name, _ in capi.Route._fields_]
    src = tmp_path / "layout.c"
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "w4a16.h"', "int main(void) {",
             '    printf("sizeof %zu\\n", sizeof(w4a16_route));']
    lines += [f'    printf("{f} %zu\\n", offsetof(w4a16_route, {f}));' for f in fields]
    tp_fields = [name for name, _ in capi.TpGroup._fields_]
    lines += ['    printf("tp_sizeof %zu\\n", sizeof(w4a16_tp_group));']
    lines += [f'    printf("tp_{f} %zu\\n", offsetof(w4a16_tp_group, {f}));' for f in tp_fields]
    lines += [f'    printf("{name} %d\\n", (int){name});' for name in capi.STATUS_NAMES.values()]
    lines += ['    printf("W4A16_FLAG_WEIGHTS_RESIDENT %d\\n", (int)W4A16_FLAG_WEIGHTS_RESIDENT);',
              '    printf("W4A16_FLAG_FP32_SCALE %d\\n", (int)W4A16_FLAG_FP32_SCALE);']
    lines += ['    printf("W4A16_OUT_F32 %d\\n", (int)W4A16_OUT_F32);',
              '    printf("W4A16_ABI_VERSION %d\\n", (int)W4A16_ABI_VERSION);', "    return 0;", "}"]
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
                    str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    assert int(out["sizeof"]) == ctypes.sizeof(capi.Route)
    assert int(out["tp_sizeof"]) == ctypes.sizeof(capi.TpGroup)
    for f in tp_fields:
        assert int(out["tp_" + f]) == getattr(capi.TpGroup, f).offset, f
    for f in fields:
        assert int(out[f]) == getattr(capi.Route, f).offset, f
    for code, name in capi.STATUS_NAMES.items():
        assert int(out[name]) == code, name
    assert int(out["W4A16_OUT_F32"]) == capi.W4A16_OUT_F32
    assert int(out["W4A16_FLAG_WEIGHTS_RESIDENT"]) == capi.W4A16_FLAG_WEIGHTS_RESIDENT
    assert int(out["W4A16_FLAG_FP32_SCALE"]) == capi.W4A16_FLAG_FP32_SCALE
    assert int(out["W4A16_ABI_VERSION"]) == capi.load().w4a16_abi_version()


@pytest.mark.skipif(__import__("shutil").which("gcc") is None, reason="needs gcc")
def test_plain_c_client_links_and_validates(tmp_path):
    """A C99 program links libw4a16.so and gets the reference's validation statuses and
    messages (kernel.cu:219-249) through the C ABI, with no Python or torch involved."""
    import subprocess
    src = tmp_path / "client.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "w4a16.h"
int main(void) {
    int bad = 0;
    if (w4a16_abi_version() != W4A16_ABI_VERSION) bad |= 1;
    /* K not a multiple of 64 */
    w4a16_status s = w4a16_validate(NULL, NULL, NULL, 1, 64, 100, 1, 64 * 100 / 8, -1);
    if (s != W4A16_ERR_K_MULTIPLE || !strstr(w4a16_last_error(), "multiple of 64")) bad |= 2;
    /* unsupported group size: K = 512 in 2 groups -> G = 256 */
    s = w4a16_validate(NULL, NULL, NULL, 1, 64, 512, 2, 64 * 512 / 8, -1);
    if (s != W4A16_ERR_GROUP_SIZE || !strstr(w4a16_last_error(), "unsupported group size")) bad |= 4;
    /* variant out of range */
    s = w4a16_validate(NULL, NULL, NULL, 1, 64, 512, 4, 64 * 512 / 8, 9);
    if (s != W4A16_ERR_VARIANT || !strstr(w4a16_last_error(), "variant")) bad |= 8;
    /* valid shape, null pointers: rejected before any device work */
    s = w4a16_gemm(NULL, NULL, NULL, NULL, 1, 64, 512, 4, 64 * 512 / 8, -1, W4A16_OUT_F16, NULL, 0, NULL);
    if (s != W4A16_ERR_NULL_POINTER) bad |= 16;
    if (strcmp(w4a16_status_string(W4A16_OK), "W4A16_OK") != 0) bad |= 32;
    printf("%d\n", bad);
    return bad;
}
''')
    exe = tmp_path / "client"
    libdir = os.path.dirname(capi.library_path())
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-L", libdir, "-lw4a16", "-Wl,-rpath," + libdir, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "0", (r.returncode, r.stdout, r.stderr)
