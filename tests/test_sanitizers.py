"""Race and memory-error detection for the host C++ runtime: the native stress
driver (csrc/tests/comm_stress.cpp) under ThreadSanitizer and under
AddressSanitizer + UndefinedBehaviorSanitizer must finish every check with no
sanitizer report."""
import pytest

from mtorus.utils import sanitize

pytestmark = pytest.mark.skipif(not sanitize.available(), reason="no C++ compiler")


@pytest.mark.parametrize("kind", ["thread", "address"])
def test_host_runtime_is_clean_under_sanitizer(kind, tmp_path):
    try:
        exe = sanitize.build(kind, str(tmp_path))
    except sanitize.SanitizerUnavailable as e:
        pytest.skip(str(e)[:200])
    code, out = sanitize.run(kind, rounds=20, exe=exe)
    assert "Sanitizer" not in out, out[-4000:]
    assert code == 0, out[-4000:]
    assert "0 failed checks" in out
