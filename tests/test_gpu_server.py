"""The policy server (behavior-2026_b200/pi05_server, openpi's WebSocket protocol over the C ABI) against
the same engine run in-process: the actions it returns for RGBA frames at 480x640 / 720x720 / 224x300
(two environments per request, one message split into continuation frames) are bit for bit what
pi05_act_batch returns for the same observation (the reference server's check: 2760/2760 actions
identical to in-process inference, π05_네이티브엔진.md:324-326); /healthz, metadata on connect,
__action_chunk_size__ and reset."""
import os
import socket
import subprocess

import numpy as np
import pytest

import wsclient

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SERVER = os.path.join(ROOT, "behavior-2026_b200", "pi05_server")
ARGS = ["--random-weights", "8", "--siglip-layers", "1", "--gemma-layers", "2", "--num-steps", "2", "--max-batch", "2",
        "--act-dim", "23", "--replan", "4", "--noise-seed", "5"]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def server(pn):
    port = _free_port()
    p = subprocess.Popen([SERVER, "--host", "127.0.0.1", "--port", str(port)] + ARGS, stdout=subprocess.PIPE,
                         stderr=subprocess.PIPE, text=True)
    line = p.stdout.readline()
    assert "listening" in line, line + p.stderr.read()
    yield port
    p.kill()
    p.wait(timeout=60)


def observation(rng, n=2):
    return {"head": rng.integers(0, 256, (n, 480, 640, 4), dtype=np.uint8),
            "left_wrist": rng.integers(0, 256, (n, 720, 720, 3), dtype=np.uint8),
            "right_wrist": rng.integers(0, 256, (n, 224, 300, 4), dtype=np.uint8),
            "tokens": rng.integers(0, 257152, (n, 200), dtype=np.int32)}


def test_healthz(server):
    assert wsclient.http_get(server, "/healthz").startswith(b"HTTP/1.1 200 OK")


def test_server_actions_equal_in_process_act_batch(pn, server):
    eng = pn.Engine(pn.Config.make(siglip_layers=1, gemma_layers=2, num_steps=2), max_batch=2)
    eng.init_random_weights(8)
    eng.set_act_config(act_dim=23, replan=4, noise_seed=5)
    rng = np.random.default_rng(3)
    cl = wsclient.Client(server)
    md = cl.metadata
    assert md["kind"] == "pi05" and md["act_dim"] == 23 and md["camera_keys"] == ["head", "left_wrist", "right_wrist"]
    keys = md["camera_keys"]
    for step in range(6):
        obs = observation(rng)
        got = cl.call(obs, fragment=1 << 20 if step % 2 else None)
        assert "error" not in got, got
        frames = [[obs[k][i] for k in keys] for i in range(2)]
        want = eng.act_batch([0, 1], frames, obs["tokens"])
        np.testing.assert_array_equal(got["action"], want, err_msg=f"step {step}")
        assert got["server_timing"]["infer_ms"] > 0
    # the next 3 actions at once; then a reset makes both environments re-plan
    obs = observation(rng)
    got = cl.call(dict(obs, __action_chunk_size__=3))
    frames = [[obs[k][i] for k in keys] for i in range(2)]
    want = np.stack([eng.act_batch([0, 1], frames, obs["tokens"]) for _ in range(3)], 1)
    np.testing.assert_array_equal(got["action"], want)
    assert cl.call({"reset": True}) == {"reset": True}
    eng.reset_slot(0)
    eng.reset_slot(1)
    obs = observation(rng)
    got = cl.call(obs)
    frames = [[obs[k][i] for k in keys] for i in range(2)]
    np.testing.assert_array_equal(got["action"], eng.act_batch([0, 1], frames, obs["tokens"]))
    # a malformed observation gets an error reply and the connection stays usable
    bad = cl.call({"head": obs["head"]})
    assert "error" in bad
    cl.close()
    eng.close()
