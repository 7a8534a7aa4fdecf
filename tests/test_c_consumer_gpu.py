"""The drop-in boundary from a C program on the GPU: tests/c_consumer/
mv4i_consumer.c, compiled with gcc against include/mv4i_b200.h and linked to
libmv4i_b200.so, runs mv4i_parse + mv4i_matvec with host buffers on every
golden case and must reproduce the reference's own mv4i_matvec output
(tests/golden/mv4i_golden.npz, written from ref/matvec_int4.c) bit for bit,
y_exp / saturation / ns included."""
import subprocess

import numpy as np
import pytest

from test_abi import build_consumer

pytestmark = pytest.mark.gpu


def _cases(golden):
    for n in range(36):
        key = "emit%d" % n
        if key + "_meta" in golden:
            m = [int(v) for v in golden[key + "_meta"]]
            yield key, golden["img%d" % m[12]].tobytes(), m
    for pre in ("lin", "sat"):
        for mode in range(3):
            key = "%s%d" % (pre, mode)
            yield key, golden[key + "_img"].tobytes(), [int(v) for v in golden[key + "_meta"]]


def test_c_consumer_matvec_matches_reference(cuda, pkg, golden, tmp_path):
    exe = build_consumer(pkg, str(tmp_path))
    n = 0
    for key, img, m in _cases(golden):
        ip, xp, op = tmp_path / "img.mv4i", tmp_path / "x.bin", tmp_path / "y.bin"
        ip.write_bytes(img)
        xp.write_bytes(np.ascontiguousarray(golden[key + "_x"], np.int16).tobytes())
        x_exp, nr, nc, mode, y_exp, sat_event, sat_count, ns = m[4], m[5], m[6], m[7], m[8], m[9], m[10], m[11]
        out = subprocess.run([exe, "matvec", str(ip), str(xp), str(x_exp), str(nr), str(nc), str(mode), str(op)],
                             capture_output=True, text=True)
        assert out.returncode == 0, (key, out.stdout, out.stderr)
        rc, ye, se, sc, nsv = [int(v) for v in out.stdout.split()]
        dt = {0: np.int16, 1: np.int32, 2: np.int64}[mode]
        y = np.frombuffer(op.read_bytes(), dt).astype(np.int64)
        assert rc == 0 and np.array_equal(y, golden[key + "_y"][:nr]), key
        assert (ye, se, sc) == (y_exp, sat_event, sat_count), key
        if mode == 0:
            assert nsv == ns, key
        n += 1
    assert n >= 40
