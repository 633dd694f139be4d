import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, 'tests', 'golden')):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a) and the built native library')


@pytest.fixture(autouse=True)
def isolated_environment(monkeypatch):
    """Tests use explicit settings, never the operator's JUDGE_* / MORJ_* environment."""
    for name in list(os.environ):
        if name.startswith(('JUDGE_', 'MORJ_')):
            monkeypatch.delenv(name)
