import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.8-flash-next_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

# achieved error margins of the GPU parity checks: (test, case, max_abs,
# rel_rms, bars); printed in the session summary, and written as JSON to
# $QMOE_MARGINS_OUT when that is set
MARGINS = []


def record_margin(case, max_abs, rel_rms, bars):
    test = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    MARGINS.append({"test": test, "case": case, "max_abs": max_abs, "rel_rms": rel_rms,
                    "bars": bars})


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not MARGINS:
        return
    terminalreporter.write_line("parity margins (max_abs, rel_rms | bars):")
    for m in MARGINS:
        terminalreporter.write_line(f"  {m['test']} [{m['case']}]: {m['max_abs']:.3e}, "
                                    f"{m['rel_rms']:.3e} | {m['bars']}")
    out = os.environ.get("QMOE_MARGINS_OUT")
    if out:
        with open(out, "w") as f:
            json.dump(MARGINS, f, indent=1)


@pytest.fixture(scope="session")
def built():
    """Builds libqmoe.so and the CPU checkers once per session."""
    import subprocess

    import oracle

    subprocess.run(["make", "-s", "-C", PKG], check=True)
    oracle.build()
    return True
