"""MiniXLA's own GPU test suite, gpu_test.c, compiled unmodified against
libminixla_b200.so (tests/dropin/gpu_test_cases.c includes it verbatim; the
oracle recipe's `dropin` target builds it from the reference sources into
oracle/_ref/).  Each case runs in its own process so a failing assert names
its case.

Every case of gpu_test.c's main() runs as written except one:
test_broadcast_bias_rejected_on_gpu (gpu_test.c:48-73) asserts that the GPU
entry points refuse a [N] bias-row ADD; this backend runs it, so
broadcast_bias_runs_on_gpu checks the same graph against execute() instead."""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

EXE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "gpu_test_cases"

# gpu_test.c's main(), in order (gpu_test.c:432-441), with the one replacement.
CASES = ["test_single_fused", "broadcast_bias_runs_on_gpu", "test_diamond_shared_input", "test_two_layer",
         "test_deep_chain", "test_module_cache", "bench_large_matmul", "test_tensorcore_correctness",
         "test_tensorcore_epilogue"]


def test_case_list_matches_the_program():
    if not EXE.exists():
        pytest.skip("oracle/_ref/gpu_test_cases not built (needs the reference sources at build time)")
    listed = subprocess.run([str(EXE)], capture_output=True, text=True, timeout=60, check=True).stdout.split()
    assert listed == CASES


@pytest.mark.parametrize("case", CASES)
def test_reference_gpu_test_case(case):
    if not EXE.exists():
        pytest.skip("oracle/_ref/gpu_test_cases not built (needs the reference sources at build time)")
    r = subprocess.run([str(EXE), case], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and f"{case} PASS" in r.stdout, f"rc={r.returncode}\n{r.stdout}\n{r.stderr}"
