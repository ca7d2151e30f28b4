"""The C interface as a C11 caller sees it (CPU only, gcc).

* Every function include/pl_attn.h declares has an inline stub with the same
  signature when the module is compiled out (-DPL_ATTN_DISABLED), as
  picolm's gpu.h stubs its backend without USE_VULKAN (gpu.h:33-42): a C11
  file binds each declared prototype to a function pointer of exactly that
  type, in both modes, with -Werror.
* The same file links against libpl_attn.so, so every declaration resolves
  to an exported definition.
* The C snippets of INTEGRATION.md compile against picolm's own model.h (the
  field names they use exist), with and without USE_PL_ATTN; skipped when
  picolm's sources are not beside this repository.
"""
import os
import re
import shutil
import subprocess

import pytest

import picolm_b200 as pb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")

pytestmark = pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not found")


def prototypes():
    """(return type, name, argument list) of each declared entry point."""
    text = open(pb.HEADER).read().split("#else /* PL_ATTN_DISABLED")[0]
    out = re.findall(r"^(int|void|const char \*)\s*(pl_\w+)\((.*?)\);", text, re.S | re.M)
    return [(r.strip(), n, " ".join(a.split())) for r, n, a in out]


def _pointer_file(tmp_path):
    lines = ["#include <stdio.h>", '#include "pl_attn.h"', ""]
    for ret, name, args in prototypes():
        lines.append(f"{ret} (*chk_{name})({args}) = {name};")
    lines.append("int main(void) {")
    lines.append("  int rc = pl_attn_init(1, 32, 4, 64, 64, 10000.f, PL_ROPE_LLAMA, 1, 0);")
    lines.append('  printf("%d %s\\n", rc, pl_attn_strerror(rc));')
    lines.append("  return 0;")
    lines.append("}")
    src = tmp_path / "abi_ptrs.c"
    src.write_text("\n".join(lines) + "\n")
    return src


def test_every_declaration_is_a_prototype():
    names = {n for _, n, _ in prototypes()}
    assert names == set(pb.declared_symbols())


def test_disabled_stubs_match_every_declaration(tmp_path):
    src = _pointer_file(tmp_path)
    exe = tmp_path / "abi_off"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-DPL_ATTN_DISABLED",
                    "-I", INCLUDE, "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    assert out.split()[0] == str(pb.PL_EDEVICE)
    assert "compiled out" in out


def test_enabled_header_links_against_the_library(tmp_path):
    from picolm_b200 import build
    build.build()
    src = _pointer_file(tmp_path)
    exe = tmp_path / "abi_on"
    libdir = os.path.dirname(pb.LIB_PATH)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", INCLUDE, "-o",
                    str(exe), str(src), "-L", libdir, "-lpl_attn", f"-Wl,-rpath,{libdir}"],
                   check=True)


# ------------------------------------------------- INTEGRATION.md snippets
def _picolm_dir():
    cand = os.environ.get("PICOLM_REF_DIR") or os.path.join(os.path.dirname(ROOT), "reference",
                                                              "picolm")
    return cand if os.path.isfile(os.path.join(cand, "model.h")) else None


def integration_snippets():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return re.findall(r"```c\n(.*?)```", text, re.S)


# what the call sites of model.c / picolm.c have in scope, as parameters of
# the wrapper function (a snippet's own declarations shadow them)
_SCOPE = ("model_t model, int l, int pos, int start_pos, int n_tokens, int dim, int n_pos, "
          "int kv_dim, float *q_batch, float *k_batch, float *v_batch, float *xb_batch, "
          "float *x_batch, float *k_tmp, float *v_tmp, uint16_t *kbuf, uint16_t *vbuf, FILE *f")


def _snippet_file(tmp_path):
    snips = integration_snippets()
    assert len(snips) >= 6
    lines = ["#include <stdio.h>", "#include <stdlib.h>", "#include <stdint.h>",
             '#include "model.h"', '#include "pl_attn.h"', ""]
    for i, body in enumerate(snips):
        body = "\n".join(ln for ln in body.splitlines() if not ln.startswith("#include"))
        lines += [f"int snippet_{i}({_SCOPE}) {{",
                  "  int rc = 0; const model_config_t *c = &model.config;",
                  "  run_state_t *s = &model.state;",
                  "  {", body, "  }", "  return rc + (c != NULL) + (s != NULL);", "}", ""]
    src = tmp_path / "snippets.c"
    src.write_text("\n".join(lines))
    return src


@pytest.mark.parametrize("mode", ["-DUSE_PL_ATTN", "-DPL_ATTN_DISABLED"])
def test_integration_snippets_compile(tmp_path, mode):
    ref = _picolm_dir()
    if ref is None:
        pytest.skip("picolm's sources (model.h) are not beside this repository")
    src = _snippet_file(tmp_path)
    subprocess.run(["gcc", "-std=c11", "-D_GNU_SOURCE", "-Wall", "-Werror",
                    "-Wno-unused-parameter", "-Wno-unused-variable", "-Wno-unused-result",
                    mode, "-I", ref, "-I", INCLUDE, "-c", "-o", str(tmp_path / "snip.o"),
                    str(src)], check=True)
