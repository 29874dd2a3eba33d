"""The drop-in shown in the reference's own model code: a tiny random-init
YANchorForCausalLM from the reference install (baseline/_ref) runs a
150-token prefill and 49 decode steps once on the reference's torch path and
once with INTEGRATION.md's patch binding this repository's CUDA ops
(tests/dropin/run_reference_model.py, a child process because it imports the
reference's pinned transformers).  Bar: logits within 2e-2, greedy ids
identical wherever the reference's top-2 margin exceeds 1e-2
(modeling_yanchor.py:392-410, :19-20, :178-313)."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_reference_model_with_b200_ops_matches_torch_path():
    import _reference
    if not _reference.available():
        pytest.skip('SKIPPED, NOT PASSED: the reference install (baseline/_ref) is absent')
    res = subprocess.run([sys.executable, os.path.join(ROOT, 'tests', 'dropin', 'run_reference_model.py')],
                         capture_output=True, text=True, timeout=900, cwd=ROOT)
    lines = [l for l in res.stdout.splitlines() if l.startswith('{')]
    assert res.returncode == 0 and lines, res.stderr[-4000:]
    r = json.loads(lines[-1])
    print(r)
    assert r['state_dict_keys_ok'] and r['bound_layers']
    assert r['prefill_max_abs'] <= 2e-2, r
    assert r['decode_max_abs'] <= 2e-2, r
    assert r['ids_compared'] > 0 and r['ids_agree'] == r['ids_compared'], r
