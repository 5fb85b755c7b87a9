"""The KERNEL_RESULT binary's output through the reference's own harness code.

``ferret_b200/ferret_kernel_result`` is the self-contained benchmark binary the
reference's agent harness runs for a task: it prints one
``KERNEL_RESULT {json}`` line (and ``KERNEL_RESULT_REFERENCE {}``).  These CPU
tests feed recorded stdout of that binary -- captured on a B200 with the
commands written in each fixture's first line, after every output row of every
configuration passed its host fp32 check -- to the reference's parser
(task_spec.py:277-328, ``parse_kernel_output`` / ``parse_reference_output``)
and scorer (task_spec.py:364-410, ``compute_score``) together with the
reference's task specs, imported from the reference tree.  They check that
every configuration the task defines is present with a valid (non-zero)
result, and that the scorer turns the line into the per-config ratios it
gates on.  Skipped when the reference tree is not available
($FERRET_REFERENCE_ROOT, else a "reference" directory beside the repository).
"""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")
REF = os.environ.get("FERRET_REFERENCE_ROOT", os.path.join(os.path.dirname(ROOT), "reference"))

TASKS = [
    ("decode", "fp8-group-gemm-dsv3-decode.yaml"),
    ("prefill", "fp8-group-gemm-dsv3-prefill.yaml"),
    ("kimi", "kimi-moe-w13-int4-grouped-gemm.yaml"),
]


@pytest.fixture(scope="module")
def task_spec():
    path = os.path.join(REF, "task_spec.py")
    if not os.path.exists(path):
        pytest.skip("reference tree not available")
    spec = importlib.util.spec_from_file_location("ferret_reference_task_spec", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod          # its dataclasses look their module up
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("task,yaml_name", TASKS)
def test_recorded_output_parses_and_scores(task_spec, task, yaml_name):
    text = open(os.path.join(GOLD, f"kernel_result_{task}.txt")).read()
    spec = task_spec.load_task_spec(os.path.join(REF, "tasks", yaml_name))
    results = task_spec.parse_kernel_output(text)
    names = [c.name for c in spec.configs]
    # every configuration of the task, each with a valid measurement (an
    # INVALID config prints 0.0)
    assert set(names) <= set(results), (names, sorted(results))
    assert all(results[n] > 0 for n in names), results
    # no scoring reference on this box (the task's baseline, DeepGEMM or
    # Marlin, is not part of this binary): the harness's ratio is then 0
    reference = task_spec.parse_reference_output(text)
    assert reference == {}
    score, ratios = task_spec.compute_score(results, reference, spec)
    assert score == 0.0 and set(ratios) == set(names)
    # with a reference present the scorer gates on result / reference
    half = {n: 2.0 * results[n] for n in names}
    score, ratios = task_spec.compute_score(results, half, spec)
    assert all(abs(r - 0.5) < 1e-12 for r in ratios.values())
    assert abs(score - 0.5) < 1e-12


def test_parser_ignores_the_reference_line_for_results(task_spec):
    out = 'x\nKERNEL_RESULT {"a": 1.5, "b": 2}\nKERNEL_RESULT_REFERENCE {"a": 3.0}\n'
    assert task_spec.parse_kernel_output(out) == {"a": 1.5, "b": 2.0}
    assert task_spec.parse_reference_output(out) == {"a": 3.0}
