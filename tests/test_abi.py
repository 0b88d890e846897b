"""The C-ABI boundary without a GPU: every function include/*.h declares is
exported by libpitorch_b200.so (a C program taking each one's address links
against the library), and the ctypes mirrors in pitorch_b200/api.py have the
C compiler's sizes and field offsets."""
import ctypes as C
import os
import re
import subprocess

import pytest

import pitorch_b200
from pitorch_b200 import api

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
HEADERS = sorted(h for h in os.listdir(INC) if h.endswith(".h"))
LIB_DIR = os.path.dirname(pitorch_b200.LIB_PATH) if hasattr(pitorch_b200, "LIB_PATH") else os.path.join(ROOT, "pitorch_b200")


def declared_functions():
    """Names of the functions the headers declare, from the preprocessed text."""
    src = "".join(f'#include "{h}"\n' for h in HEADERS)
    out = subprocess.run(["gcc", "-E", "-P", "-I", INC, "-x", "c", "-"], input=src, capture_output=True,
                         text=True, check=True).stdout
    # drop struct bodies and typedefs of function pointers, then take "name(" at statement level
    out = re.sub(r"\{[^{}]*\}", "", out)
    names = set()
    for stmt in out.split(";"):
        stmt = " ".join(stmt.split())
        if stmt.startswith("typedef") or "(" not in stmt:
            continue
        m = re.match(r"^(?:extern )?[\w\s\*]+?\**\s*\b((?:pt|ptc)_\w+)\s*\(", stmt)
        if m:
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_api():
    names = declared_functions()
    for must in ("pt_pi_init", "pt_pi_init_shard", "pt_forward_step", "pt_train_step", "pt_generate",
                 "pt_dist_setup", "pt_dist_forward_step", "pt_dist_train_step", "ptc_matvec",
                 "ptc_sgemm", "ptc_sgemm_noalloc", "pt_encode", "pt_sample"):
        assert must in names, must
    assert len(names) > 100


def test_library_exports_every_declared_function(tmp_path):
    names = declared_functions()
    lib = pitorch_b200.lib()  # builds nothing; raises if the library is missing
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and a C caller links: take the address of each through the headers' own prototypes
    src = tmp_path / "link.c"
    src.write_text("".join(f'#include "{h}"\n' for h in HEADERS) +
                   "void *syms[] = {\n" + ",\n".join(f"(void *){n}" for n in names) + "\n};\n"
                   "int main(void) { return syms[0] == 0; }\n")
    so = lib._name
    r = subprocess.run(["gcc", "-I", INC, str(src), so, f"-Wl,-rpath,{os.path.dirname(so)}",
                        "-o", str(tmp_path / "link")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


STRUCTS = {
    "pt_config_t": api.pt_config_t, "pt_weights_t": api.pt_weights_t, "pt_state_t": api.pt_state_t,
    "pt_activations_t": api.pt_activations_t, "pt_grads_t": api.pt_grads_t,
    "pt_backward_buf_t": api.pt_backward_buf_t, "pt_context_t": api.pt_context_t,
    "pt_shard_info_t": api.pt_shard_info_t, "pt_dist_t": api.pt_dist_t,
    "pt_dist_result_t": api.pt_dist_result_t, "pt_token_index_t": api.pt_token_index_t,
    "pt_tokenizer_t": api.pt_tokenizer_t, "pt_sampler_t": api.pt_sampler_t,
}


def test_ctypes_layouts_match_c(tmp_path):
    lines = ["#include <stdio.h>", "#include <stddef.h>"] + [f'#include "{h}"' for h in HEADERS]
    lines.append("int main(void) {")
    for cname, cls in STRUCTS.items():
        lines.append(f'  printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'  printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("  return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", INC, str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.split("\n") if l)
    for cname, cls in STRUCTS.items():
        assert int(got[cname]) == C.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, (cname, f)
