import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU; run with -m gpu on a GPU box")


def pytest_terminal_summary(terminalreporter):
    """Tier-2 id parity: how many tokens per case were excused by a near tie."""
    from tests import helpers

    if helpers.EXCUSED:
        terminalreporter.write_sep("-", "tier-2 near-tie tokens excused (case: excused / tokens)")
        for case, (n, tokens) in sorted(helpers.EXCUSED.items()):
            terminalreporter.write_line(f"{case}: {n} / {tokens}")
