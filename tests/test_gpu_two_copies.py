"""Two copies of the library loaded into one process (say, two frameworks
that each ship it, or a plugin that is reloaded under a new file name): each
copy carries its own statically linked CUDA runtime, and both must launch and
agree.  The copies run in a child process (tests/two_copies_worker.py) so that
the second copy stays out of the test process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_two_copies_in_one_process():
    r = subprocess.run(["timeout", "-k", "30", "300", sys.executable,
                        os.path.join(HERE, "two_copies_worker.py")],
                       capture_output=True, text=True, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
