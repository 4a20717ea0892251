"""CPU tests of the C-ABI boundary: the library loads, exports every symbol
the header declares, and its struct layouts are the reference's."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from minixla_b200 import abi
from minixla_b200 import lib as mlib
from oracle.refdir import ref_dir

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "minixla_b200.h"
REF = ref_dir() or ROOT / "baseline" / "_ref"
DROPIN_APP = ROOT / "oracle" / "_ref" / "dropin_app"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^MXB_API\s+[\w\s\*]+?\b(\w+)\s*\(", text, flags=re.M)))


def test_header_declares_reference_entry_points():
    names = declared_symbols()
    for ref_name in ["gpu_ctx_create", "gpu_ctx_destroy", "gpu_execute", "gpu_time_kernel_ms",
                     "gpu_run_tensorcore", "gpu_time_kernel_tc_ms", "gpu_run_fused"]:
        assert ref_name in names


def test_library_loads_and_exports_every_declared_symbol():
    lib = mlib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared_symbols()) == set(mlib.PROTOTYPES), "ctypes prototypes out of sync with the header"


def test_exports_nothing_undeclared():
    out = subprocess.run(["nm", "-D", "--defined-only", str(mlib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_symbols())


def test_ctypes_mirror_layout():
    assert C.sizeof(abi.Tensor) == 40 and C.sizeof(abi.Node) == 64 and C.sizeof(abi.EpStep) == 16
    assert abi.Node.n_epilogue.offset == 56 and abi.Node.epilogue.offset == 48 and abi.Node.is_const.offset == 44
    assert abi.Tensor.size.offset == 32 and abi.Tensor.ndim.offset == 24


def test_error_paths_without_gpu_or_with_bad_args():
    lib = mlib.load()
    # NULL arguments are rejected with a message, never a crash.
    assert not lib.gpu_execute(None, None)
    assert lib.gpu_time_kernel_ms(None, None, 1, 1) == -1.0
    assert lib.gpu_ctx_set_precision(None, 7) == -1
    assert lib.mxb_fused_gemm(None, None, 0, None, 0, None, 0, 1, 1, 1, None, 0, 1, None) == mlib.MXB_E_ARG
    assert mlib.last_error()


_LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include HDR
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\n", sizeof(Tensor), offsetof(Tensor, data), offsetof(Tensor, shape),
         offsetof(Tensor, strides), offsetof(Tensor, ndim), offsetof(Tensor, size));
  printf("%zu %zu %zu\n", sizeof(EpStep), offsetof(EpStep, op), offsetof(EpStep, operand));
  printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(Node), offsetof(Node, op),
         offsetof(Node, inputs), offsetof(Node, n_inputs), offsetof(Node, output), offsetof(Node, owns_output),
         offsetof(Node, visited), offsetof(Node, uses), offsetof(Node, is_const), offsetof(Node, epilogue),
         offsetof(Node, n_epilogue));
  printf("%d %d %d\n", (int)OP_INPUT, (int)OP_RELU, (int)OP_FUSED);
  return 0;
}
"""


def _probe(tmp_path, header, tag):
    src = tmp_path / f"probe_{tag}.c"
    src.write_text(_LAYOUT_PROBE.replace("HDR", f'"{header}"'))
    exe = tmp_path / f"probe_{tag}"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    return subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout


@pytest.mark.skipif(not (REF / "graph.h").exists(), reason="reference headers not present")
def test_layout_matches_reference_headers(tmp_path):
    ours = _probe(tmp_path, HEADER, "ours")
    theirs = _probe(tmp_path, REF / "graph.h", "ref")
    assert ours == theirs


@pytest.mark.skipif(not (REF / "gpu_exec.h").exists(), reason="reference headers not present")
def test_header_compiles_after_reference_headers(tmp_path):
    """A MiniXLA program including gpu_exec.h / runtime.h first, then this header."""
    src = tmp_path / "mix.c"
    src.write_text(f'#include "{REF}/gpu_exec.h"\n#include "{REF}/runtime.h"\n#include "{HEADER}"\n'
                   "int main(void) { GpuCtx* c = gpu_ctx_create_on(0); gpu_ctx_set_precision(c, "
                   "GPU_PRECISION_TF32); return c == 0; }\n")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-c", str(src), "-o", str(tmp_path / "mix.o")],
                   check=True)


@pytest.mark.skipif(not (REF / "graph.c").exists(), reason="reference sources not present")
def test_reference_c_program_links_as_drop_in(tmp_path):
    """A MiniXLA C program (tests/dropin/dropin_app.c), unchanged headers and
    graph code, links against libminixla_b200.so in place of gpu_exec.c /
    runtime.c / ptx.c and, where no GPU exists, fails gracefully."""
    exe = tmp_path / "app"
    lib_dir = mlib.LIB_PATH.parent
    subprocess.run(["gcc", "-O2", "-I", str(REF), "-o", str(exe), str(ROOT / "tests" / "dropin" / "dropin_app.c"),
                    str(REF / "graph.c"), str(REF / "tensor.c"), str(REF / "optimizer.c"), "-L", str(lib_dir),
                    "-lminixla_b200", f"-Wl,-rpath,{lib_dir}", "-lm"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    import torch

    if torch.cuda.is_available():
        assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
    else:
        assert r.returncode == 2 and "no GPU context" in r.stdout


@pytest.mark.gpu
def test_reference_c_program_runs_on_gpu():
    """The same C program, prebuilt against the library by the oracle recipe
    (`make -C oracle dropin`), run on the GPU: gpu_execute gives tests.c's
    answer {0, 28, 49, 0}."""
    if not DROPIN_APP.exists():
        pytest.skip("oracle/_ref/dropin_app not built (needs the reference sources at build time)")
    r = subprocess.run([str(DROPIN_APP)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
