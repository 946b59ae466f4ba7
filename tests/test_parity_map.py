"""The parity table covers the reference's whole test inventory and names only
tests that exist here."""
import importlib
import os
import sys

from parity_map import PARITY

HERE = os.path.dirname(os.path.abspath(__file__))


def test_parity_map_covers_the_reference_inventory():
    assert len(PARITY) == 292  # reference test functions
    assert sum(n for _, _, n, _ in PARITY) == 313  # with the rstest cases
    keys = [(f, name) for f, name, _, _ in PARITY]
    assert len(set(keys)) == len(keys)
    assert all(tests for *_, tests in PARITY)


def test_every_mapped_test_exists():
    if HERE not in sys.path:
        sys.path.insert(0, HERE)
    missing = []
    for *_, tests in PARITY:
        for t in tests:
            mod, fn = t.split("::")
            m = importlib.import_module(mod[:-3])
            if not callable(getattr(m, fn, None)):
                missing.append(t)
    assert not missing, missing
