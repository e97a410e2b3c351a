"""NVTX tracing of the entry points: off by default (the functions are the
undecorated ones), on with CQ_NVTX=1 at import, where every call is one
balanced push/pop pair named after the entry point.  Host-only: the NVTX
calls are recorded by a stand-in, so no GPU is needed."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tracing_off_by_default():
    env = {k: v for k, v in os.environ.items() if k != "CQ_NVTX"}
    code = ("import chronoquant_mlx_b200 as c\n"
            "assert not hasattr(c.chronoquant_sdpa, '__cq_trace__')\n"
            "assert not hasattr(c.ChronoQuantCache.update_and_fetch, '__cq_trace__')\n"
            "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


def test_tracing_ranges_are_balanced():
    code = r"""
import torch
calls = []
torch.cuda.nvtx.range_push = lambda name: calls.append(("push", name))
torch.cuda.nvtx.range_pop = lambda: calls.append(("pop",))
import chronoquant_mlx_b200 as c
from chronoquant_mlx_b200.trace import traced
names = {c.chronoquant_sdpa.__cq_trace__, c.ChronoQuantCache.update_and_fetch.__cq_trace__,
         c.ChronoQuantCache.reconstruct_history.__cq_trace__}
assert names == {"cq.sdpa", "cq.append", "cq.reconstruct"}, names

@traced("cq.test")
def f(x):
    if x < 0:
        raise ValueError("negative")
    return 2 * x

assert f(3) == 6
try:
    f(-1)
except ValueError:
    pass
assert calls == [("push", "cq.test"), ("pop",), ("push", "cq.test"), ("pop",)], calls
print("ok")
"""
    env = dict(os.environ, CQ_NVTX="1")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]
