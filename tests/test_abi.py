"""The C-ABI library loads without a GPU and exports exactly what include/*.h declares.

No compute is launched here: the only calls are argument-validation paths
that return before touching the CUDA runtime.
"""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        text = h.read_text()
        names |= set(re.findall(r"^AMP_API\s+[\w\s\*]+?\b(amp_\w+)\s*\(", text, flags=re.M))
        # the plugin contract declares its symbol through a typedef + name macro
        names |= set(re.findall(r'#define\s+AMP_PLUGIN_\w+_SYMBOL\s+"(\w+)"', text))
    return names


def exported_symbols(lib: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True,
                         text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_header_symbols_are_exported(amp_lib):
    import amp_b200
    decl = declared_symbols()
    assert decl, "no declarations parsed"
    exp = exported_symbols(amp_b200.LIB_PATH)
    missing = decl - exp
    assert not missing, f"declared but not exported: {sorted(missing)}"
    extra = {s for s in exp if s.startswith("amp_")} - decl
    assert not extra, f"exported but not declared: {sorted(extra)}"


def test_python_signature_table_covers_header(amp_lib):
    from amp_b200._lib import SIGNATURES
    assert set(SIGNATURES) == declared_symbols()
    for name in SIGNATURES:
        assert hasattr(amp_lib, name)


def test_library_is_sm100a_only_and_has_no_cpu_path(amp_lib):
    import amp_b200
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", str(amp_b200.LIB_PATH)],
                         capture_output=True, text=True).stdout
    assert "sm_100a" in out
    assert "sm_90" not in out and "sm_80" not in out


def test_argument_errors_return_before_cuda(amp_lib):
    from amp_b200._lib import call, AmpError
    with pytest.raises(AmpError) as e:
        call("amp_fp8_quant_e4m3_dev", None, -1, None, None, None, None, 0, None)
    assert e.value.code == -1
    with pytest.raises(AmpError) as e:
        call("amp_fp8_dequant_e4m3_dev", None, 5, None, None, None)
    assert e.value.code == -1
    # workspace smaller than the declared requirement is rejected
    need = amp_lib.amp_fp8_quant_workspace_bytes(1 << 26)
    assert need >= 4
    buf = C.create_string_buffer(16)
    with pytest.raises(AmpError):
        call("amp_fp8_quant_e4m3_dev", C.addressof(buf), 0, None, C.addressof(buf), None,
             C.addressof(buf), need - 4, None)
    assert b"workspace" in amp_lib.amp_last_error()


def test_abi_version(amp_lib):
    assert amp_lib.amp_abi_version() >= 100


@pytest.mark.parametrize("header", sorted(p.name for p in (ROOT / "include").glob("*.h")))
@pytest.mark.parametrize("lang", [["gcc", "-std=c99", "-pedantic", "-x", "c"],
                                  ["g++", "-std=c++11", "-x", "c++"]])
def test_headers_compile_as_c_and_cxx(header, lang):
    """The boundary is a C ABI: each header stands alone in strict C and in C++."""
    r = subprocess.run([*lang, "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                        str(ROOT / "include" / header)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


LOADER = r"""
#include <dlfcn.h>
#include <stdio.h>
#include "amp_plugin.h"
int main(int argc, char** argv) {
    void* h = dlopen(argv[1], RTLD_NOW);          /* as amp_validate_kernel loads plugins */
    if (!h) { fprintf(stderr, "%s\n", dlerror()); return 2; }
    amp_user_gemm_fp32_fn fn = (amp_user_gemm_fp32_fn)dlsym(h, AMP_PLUGIN_GEMM_FP32_SYMBOL);
    if (!fn) { fprintf(stderr, "%s\n", dlerror()); return 3; }
    return 0;
}
"""


def test_plugin_resolves_through_amps_loader_contract(amp_lib, tmp_path):
    """A plain-C host with no CUDA linked resolves the plugin symbol through
    the header's typedef and name macro after dlopen(RTLD_NOW); nothing is called."""
    import amp_b200
    src = tmp_path / "loader.c"
    src.write_text(LOADER)
    exe = tmp_path / "loader"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(src), "-o", str(exe), "-ldl"], check=True)
    r = subprocess.run([str(exe), str(amp_b200.LIB_PATH)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
