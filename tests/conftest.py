import json
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def golden_cases(index="index.json"):
    """The reference's XGBoost 3.4.1 fixture cases (tests/golden/<index>)."""
    out = []
    for c in json.loads((GOLDEN / index).read_text())["cases"]:
        n, F = c["n_rows"], c["n_features"]
        X = np.fromfile(GOLDEN / f"{c['name']}.x", dtype="<f4").reshape(n, F)
        y = np.fromfile(GOLDEN / f"{c['name']}.y", dtype="<f4")
        m = np.fromfile(GOLDEN / f"{c['name']}.margin", dtype="<f4")
        w = None
        if c.get("weights"):
            w = np.fromfile(GOLDEN / f"{c['name']}.w", dtype="<f4")
        params = dict(objective=c["objective"], max_depth=c["max_depth"], num_boost_round=c["n_rounds"],
                      max_bin=c["max_bin"], eta=c["eta"], reg_lambda=c["lambda"], gamma=c["gamma"],
                      min_child_weight=c["min_child_weight"], base_score=c["base_score"])
        if "monotone_constraints" in c:
            params["monotone_constraints"] = c["monotone_constraints"]
        out.append((c["name"], X, y, w, m, params))
    return out


@pytest.fixture(scope="session")
def oracle():
    from oracle import RefCPU
    return RefCPU()
