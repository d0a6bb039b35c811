"""The policy server's wire formats on the CPU (no engine is created): SHA-1, base64 and the RFC 6455
Sec-WebSocket-Accept example, msgpack with openpi's array packing (pi05_server --selftest), and the
command line's refusal of incomplete options."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SERVER = os.path.join(ROOT, "behavior-2026_b200", "pi05_server")


def test_server_wire_selftest(pn):
    r = subprocess.run([SERVER, "--selftest"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "selftest ok" in r.stdout, r.stdout + r.stderr


def test_server_needs_weights_or_a_seed(pn):
    r = subprocess.run([SERVER, "--port", "1"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "--weights" in r.stderr
