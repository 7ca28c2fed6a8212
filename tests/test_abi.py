"""The C ABI without a GPU: the library loads, exports every function the
headers in include/ declare, validates arguments on the host, and the drop-in
headers build a reference server unmodified."""
import ctypes as C
import os
import re
import subprocess

import pytest

import lal_b200
from lal_b200 import LalTailError

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
HEADERS = [os.path.join(INCLUDE, "lal_tail.h"),
           os.path.join(INCLUDE, "runtime", "lal_q8_kernel.h"),
           os.path.join(INCLUDE, "runtime", "lal_sampling.h")]
# the samaidev/lal checkout: $LAL_REF, else a sibling of this repository
# named "reference" (as oracle/Makefile assumes)
REF = os.environ.get("LAL_REF", os.path.join(os.path.dirname(ROOT), "reference"))


def declared_functions():
    names = set()
    for hdr in HEADERS:
        src = open(hdr).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(lal_\w+)\s*\(", src, re.M):
            if "typedef" in src[max(0, m.start() - 40):m.start() + 1]:
                continue
            names.add(m.group(1))
    # static helpers kept inline in the drop-in header
    names.discard("lal_sampling_init")
    return names


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", lal_b200.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_loads_and_reports_version():
    v = lal_b200.lib().lal_tail_version().decode()
    assert "sm_100a" in v


def test_every_declared_function_is_exported():
    decl = declared_functions()
    assert len(decl) >= 35
    missing = decl - exported_symbols()
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_exports_are_exactly_the_declared_abi():
    extra = exported_symbols() - declared_functions()
    assert not extra, f"exported but undeclared: {sorted(extra)}"


def test_python_mirror_binds_every_export():
    assert exported_symbols() <= set(lal_b200.SIGNATURES)


def test_create_rejects_bad_config_on_the_host():
    with pytest.raises(LalTailError) as e:
        lal_b200.DecodeTail(vocab_size=0, n_embd=16)
    assert e.value.code == 1
    with pytest.raises(LalTailError) as e:
        lal_b200.DecodeTail(vocab_size=100, n_embd=16, shard_rank=2, shard_count=2)
    assert e.value.code == 1


def test_drop_in_headers_compile_standalone(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#define XQ_MAX 4096\n#include "runtime/lal_q8_kernel.h"\n'
                   '#include "runtime/lal_sampling.h"\n'
                   "int main(void){ LalRecentTokens r = {{0}, 0}; lal_recent_push(&r, 3);\n"
                   " return r.n == 1 ? 0 : 1; }\n")
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-Wall", "-Werror", "-Wno-unused-variable", "-Wno-unused-function",
                    f"-I{INCLUDE}", str(src), "-o", str(exe),
                    f"-L{os.path.dirname(lal_b200.LIB_PATH)}", "-llal_tail",
                    f"-Wl,-rpath,{os.path.dirname(lal_b200.LIB_PATH)}"], check=True)
    # lal_recent_push is host bookkeeping: runs without a GPU
    assert subprocess.run([str(exe)]).returncode == 0


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "tools/server/qwen7b_server.c")),
                    reason="reference checkout absent")
def test_unmodified_qwen7b_server_links_against_the_drop_ins(tmp_path):
    exe = tmp_path / "qwen7b_server"
    subprocess.run(["gcc", "-O1", "-mavx2", "-mfma", "-mf16c", "-fopenmp", "-w",
                    f"-I{INCLUDE}", f"-I{REF}", os.path.join(REF, "tools/server/qwen7b_server.c"),
                    "-o", str(exe), f"-L{os.path.dirname(lal_b200.LIB_PATH)}", "-llal_tail",
                    "-lm", "-ldl"], check=True)
    und = subprocess.run(["nm", str(exe)], capture_output=True, text=True).stdout
    for sym in ("lal_quantize_x_int8", "lal_compute_abs_xq", "lal_lm_head_int8_range_abs",
                "lal_quantize_q8_per_row"):
        assert re.search(rf"\bU {sym}\b", und), sym


def test_recent_push_matches_reference_fifo():
    rt = lal_b200.RecentTokens()
    for t in range(300):
        lal_b200.lib().lal_recent_push(C.byref(rt), t)
    assert rt.n == 256
    assert list(rt.tokens) == list(range(44, 300))
