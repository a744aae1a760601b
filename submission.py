"""MegaBench-loadable submission: `python -m megabench evaluate --submission <repo>/submission.py`.

The harness imports this file by path and calls build(case) (megabench/harness/runner.py:53-69); the
implementation lives in kimi_k3_goalbox_b200.submission.
"""

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from kimi_k3_goalbox_b200.submission import Runner, build  # noqa: E402,F401
