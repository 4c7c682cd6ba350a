"""The cross-host hop (rtc.js frames over TCP, pipeline.js:226-253): frame round
trips through TcpTransport and FrameServer, failures surfacing as errors, and (on
a GPU) a two-stage LeaderPipeline decoding the same tokens as one stage."""
import socket

import numpy as np
import pytest

from helpers import build_leader, get_weights, load_stage_weights, model_config, oracle_cfg


def echo_stage(dllm):
    """A stand-in stage host: adds 1 to every value and replies RESP with posStart + n rows."""
    F = dllm.FRAME

    def handler(data):
        fr = dllm.frames.unpack(data)
        out = fr["f32"] + 1.0
        if fr["msgType"] == F["FINAL_REQ"]:
            out = out[-4:]
        return dllm.frames.pack(F["RESP"], fr["seqId"], fr["posStart"] + 1, out)
    return handler


def test_tcp_frames_round_trip(dllm):
    srv = dllm.FrameServer(echo_stage(dllm)).start()
    tr = dllm.TcpTransport({7: ("127.0.0.1", srv.port)})
    try:
        F = dllm.FRAME
        for seq, n in ((1, 12), (2, 1 << 18), (3, 4)):  # small, 1 MiB, small on the same connection
            x = np.random.default_rng(seq).standard_normal(n).astype(np.float32)
            resp = dllm.frames.unpack(tr(7, dllm.frames.pack(F["HIDDEN_REQ"], seq, 40, x)))
            assert resp["msgType"] == F["RESP"] and resp["seqId"] == seq and resp["posStart"] == 41
            np.testing.assert_array_equal(resp["f32"], x + 1.0)
        resp = dllm.frames.unpack(tr(7, dllm.frames.pack(F["FINAL_REQ"], 9, 0, np.zeros(8, np.float32))))
        assert resp["f32"].size == 4
    finally:
        tr.close()
        srv.stop()


def test_tcp_handler_failure_raises(dllm):
    def bad(data):
        raise RuntimeError("stage failed")
    srv = dllm.FrameServer(bad).start()
    tr = dllm.TcpTransport({0: ("127.0.0.1", srv.port)}, timeout=5.0)
    try:
        with pytest.raises((ConnectionError, OSError)):
            tr(0, dllm.frames.pack(dllm.FRAME["HIDDEN_REQ"], 1, 0, np.zeros(4, np.float32)))
    finally:
        tr.close()
        srv.stop()


def test_tcp_no_peer_raises(dllm):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()  # nothing listens there
    tr = dllm.TcpTransport({0: ("127.0.0.1", port)}, timeout=2.0)
    with pytest.raises(OSError):
        tr(0, dllm.frames.pack(dllm.FRAME["HIDDEN_REQ"], 1, 0, np.zeros(4, np.float32)))


def test_bad_frame_size_rejected(dllm):
    with pytest.raises(ValueError):
        dllm.frames.unpack(b"\x00" * 18)  # rtc.js:17


def test_oversized_frame_closes_connection(dllm):
    """A length prefix beyond MAX_FRAME_BYTES makes the server drop the connection
    (no exception escapes its thread); the server keeps serving new connections."""
    import struct
    srv = dllm.FrameServer(echo_stage(dllm)).start()
    try:
        s = socket.create_connection(("127.0.0.1", srv.port), timeout=5.0)
        s.sendall(struct.pack("<Q", dllm.net.MAX_FRAME_BYTES + 1))
        assert s.recv(16) == b""  # closed by the server
        s.close()
        tr = dllm.TcpTransport({0: ("127.0.0.1", srv.port)}, timeout=5.0)
        x = np.arange(8, dtype=np.float32)
        resp = dllm.frames.unpack(tr(0, dllm.frames.pack(dllm.FRAME["HIDDEN_REQ"], 2, 0, x)))
        np.testing.assert_array_equal(resp["f32"], x + 1.0)
        tr.close()
    finally:
        srv.stop()


@pytest.mark.gpu
@pytest.mark.parametrize("via", ["local", "tcp"])
def test_two_stage_leader_matches_single_node(dllm, weights_cache, via):
    """Leader owns layers [0, 1) + head; a second Stage owns [1, 2) behind the
    transport. Greedy tokens equal the oracle's generate (pipeline.js:255-281 on
    the CPU restatement) and the single-node generate."""
    import ref_forward as ref
    cfg = oracle_cfg("tiny")
    W = get_weights(weights_cache, "tiny", cfg)
    prompt, steps = [11, 200, 37, 5], 6
    oracle_tokens, _ = ref.OracleLeader(cfg, ref.Weights(W), "f32").generate(prompt, steps)
    ctx1, single = build_leader(dllm, cfg, W, "f32")
    want = []
    single.onToken = want.append
    single.generate(prompt, steps)
    single.close()
    ctx1.close()

    ctx = dllm.initKernels(0, model_config(dllm, cfg, "f32"))
    remote = dllm.Stage(ctx, 1, 2)
    load_stage_weights(ctx, remote, W, 1, 2)
    srv, transport = None, dllm.LocalTransport({1: remote})
    if via == "tcp":
        srv = dllm.serve_stage(remote)
        transport = dllm.TcpTransport({1: ("127.0.0.1", srv.port)})
    ld = dllm.LeaderPipeline(ctx, (0, 1), stages=[{"id": 0, "start": 0, "end": 1}, {"id": 1, "start": 1, "end": 2}],
                             opts={"myId": 0, "transport": transport})
    load_stage_weights(ctx, ld.stage, W, 0, 1)
    ld.loadLeaderWeights(W["model.embed_tokens.weight"], W["model.norm.weight"], W.get("lm_head.weight"))
    got = []
    ld.onToken = got.append
    ld.generate(prompt, steps)
    try:
        assert got == list(oracle_tokens)
        assert got == want
        assert remote.T0 == len(prompt) + steps - 1
    finally:
        if srv is not None:
            transport.close()
            srv.stop()
        ld.close()
        remote.close()
        ctx.close()
