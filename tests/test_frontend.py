"""The faster front-end passes (``ad_b200.frontend``) give the reference's
own proc.  Needs the reference project (``AD_REFERENCE`` = its checkout):
each case is traced twice by ``tests/golden/gen_fixtures.py``, once with the
reference's unchanged passes and once with ``frontend.install()``, and the
two procs must be equal (same commands, ids, kernel args, order)."""
import gzip
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("AD_REFERENCE", "")


def _trace(case, mode, out):
    env = dict(os.environ, AD_LINEARIZE=mode, AD_FIXTURE_OUT=str(out))
    subprocess.run([sys.executable, os.path.join(HERE, "golden", "gen_fixtures.py"), case],
                   env=env, check=True, capture_output=True, timeout=600)
    with gzip.open(os.path.join(out, f"{case}.json.gz")) as f:
        return json.load(f)["proc"]


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "autodiff")), reason="AD_REFERENCE not set")
@pytest.mark.parametrize("case", ["mlp", "lnsm_64_256", "dotsig_128", "concat",
                                  "encdy_1_2_16_32_2_64_3", "encdy_2_4_16_32_4_64_1"])
def test_fast_frontend_gives_reference_proc(case, tmp_path):
    fast = _trace(case, "fast", tmp_path / "fast")
    ref = _trace(case, "reference", tmp_path / "ref")
    assert fast == ref
