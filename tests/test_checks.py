"""The bounds-checked debug build (``build.py --checks`` ->
libchronoquant_b200_checks.so, loaded when CQ_CHECKS=1 is set at import).

CPU: the variable selects that library and it exports every entry point.
GPU (in a subprocess, so the release library of this process is not
replaced): the checks build gives bit-identical cache bytes, attention and
reconstruction, records no error on valid input, and turns a page index
outside the pool into device error 7 rather than following it.  The bad
index is made by shrinking the descriptor's pool size (n_pages = 1) over a
cache that really holds three pages, so every page the kernels could reach
is still inside the real allocation."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKS_LIB = os.path.join(ROOT, "chronoquant_mlx_b200", "libchronoquant_b200_checks.so")

WORKER = r"""
import ctypes, math, os, sys
import numpy as np
import torch
sys.path.insert(0, os.getcwd())
from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa, _lib
from chronoquant_mlx_b200._tensors import cq_dtype, stream_ptr
from oracle import cq_oracle as O
out_dir = sys.argv[1]
dev = torch.device("cuda")
lib = _lib.lib()
print("lib", os.path.basename(_lib.LIB_PATH))
K, V = O.ar1_kv(1, 2, 600, 128, seed=4)
c = ChronoQuantCache(stride_k=32, stride_v=8, dead_zone_v=0.0)
c.update_and_fetch(torch.from_numpy(K).to(dev).half(), torch.from_numpy(V).to(dev).half())
g = torch.Generator(device="cpu").manual_seed(2)
q = (torch.randn((1, 8, 1, 128), generator=g) / math.sqrt(128)).to(torch.bfloat16).to(dev)
o = chronoquant_sdpa(q, None, None, c, 1.0 / math.sqrt(128))
kk, vv = c.reconstruct_history()
torch.cuda.synchronize()
np.save(os.path.join(out_dir, "o.npy"), o.float().cpu().numpy())
np.save(os.path.join(out_dir, "k.npy"), kk.cpu().numpy())
np.save(os.path.join(out_dir, "buf.npy"), c.store.buf.cpu().numpy())
code = ctypes.c_int(0)
_lib.check(lib.cq_device_error(ctypes.byref(code), 1))
print("valid", code.value)
# a descriptor whose pool claims one page, over a block table that maps pages 0..2
desc = c.store.descriptor()
bad = type(desc).from_buffer_copy(desc)
bad.n_pages = 1
T = c.offset
rec = torch.empty((1, 2, T, 128), dtype=torch.float16, device=dev)
_lib.check(lib.cq_reconstruct(ctypes.byref(bad), 0, T, rec.data_ptr(), 0, stream_ptr(dev)))
torch.cuda.synchronize()
_lib.check(lib.cq_device_error(ctypes.byref(code), 1))
print("reconstruct", code.value)
ln = torch.tensor([T, 0], dtype=torch.int64, device=dev)
need = ctypes.c_size_t(0)
_lib.check(lib.cq_attention_workspace(ctypes.byref(bad), T, 8, 1, 0, ctypes.byref(need)))
ws = torch.zeros(max(1, (need.value + 3) // 4), dtype=torch.float32, device=dev)
qq = q.reshape(1, 8, 128)
out = torch.empty((1, 8, 128), dtype=torch.float32, device=dev)
_lib.check(lib.cq_attention_at(ctypes.byref(bad), ln.data_ptr(), T, qq.data_ptr(), cq_dtype(qq), 8, qq.stride(0),
                               qq.stride(1), 1.0 / math.sqrt(128), out.data_ptr(), cq_dtype(out), None, ws.data_ptr(),
                               ws.numel() * 4, stream_ptr(dev)))
torch.cuda.synchronize()
_lib.check(lib.cq_device_error(ctypes.byref(code), 1))
print("attention", code.value)
o2 = chronoquant_sdpa(q, None, None, c, 1.0 / math.sqrt(128))  # the context is still usable
torch.cuda.synchronize()
_lib.check(lib.cq_device_error(ctypes.byref(code), 1))
print("after", code.value, bool(torch.equal(o2, o)))
"""


def test_checks_build_selected_and_complete():
    if not os.path.exists(CHECKS_LIB):
        pytest.skip("checks library not built (python -m chronoquant_mlx_b200.build --checks)")
    code = ("import ctypes, os\n"
            "import chronoquant_mlx_b200._lib as L\n"
            "assert os.path.basename(L.LIB_PATH) == 'libchronoquant_b200_checks.so', L.LIB_PATH\n"
            "l = ctypes.CDLL(L.LIB_PATH)\n"
            "missing = [n for n in L.EXPORTED if not hasattr(l, n)]\n"
            "assert not missing, missing\n"
            "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=dict(os.environ, CQ_CHECKS="1"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


@pytest.mark.gpu
def test_checks_build_matches_release_and_reports_bad_pages(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert os.path.exists(CHECKS_LIB), "checks library not built"
    r = subprocess.run([sys.executable, "-c", WORKER, str(tmp_path)], cwd=ROOT, env=dict(os.environ, CQ_CHECKS="1"),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    lines = dict(l.split(" ", 1) for l in r.stdout.strip().splitlines())
    assert lines["lib"] == "libchronoquant_b200_checks.so"
    assert lines["valid"] == "0"
    assert lines["reconstruct"] == "7" and lines["attention"] == "7", r.stdout
    assert lines["after"] == "0 True", r.stdout

    # the same computation with this process's release library
    import math
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa
    from oracle import cq_oracle as O
    dev = torch.device("cuda")
    K, V = O.ar1_kv(1, 2, 600, 128, seed=4)
    c = ChronoQuantCache(stride_k=32, stride_v=8, dead_zone_v=0.0)
    c.update_and_fetch(torch.from_numpy(K).to(dev).half(), torch.from_numpy(V).to(dev).half())
    g = torch.Generator(device="cpu").manual_seed(2)
    q = (torch.randn((1, 8, 1, 128), generator=g) / math.sqrt(128)).to(torch.bfloat16).to(dev)
    o = chronoquant_sdpa(q, None, None, c, 1.0 / math.sqrt(128))
    kk, _ = c.reconstruct_history()
    assert np.array_equal(np.load(tmp_path / "buf.npy"), c.store.buf.cpu().numpy())
    assert np.array_equal(np.load(tmp_path / "k.npy"), kk.cpu().numpy())
    assert np.array_equal(np.load(tmp_path / "o.npy"), o.float().cpu().numpy())
