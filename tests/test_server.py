"""The HTTP front end (the reference's src/app/Opure_Server.cpp routes over this engine).

CPU: the /generate body parser, and the routing, status codes and request framing of a
server started with no engine (sockets on 127.0.0.1 only). GPU: one /generate on a
one-engine server returns the oracle's greedy tokens, and /metrics reports it.
"""
import http.client
import json
import os

import numpy as np
import pytest

import oracle
from voxelengine import engine as ve


def request(port, method, path, body=None, headers=None):
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=60)
    try:
        c.request(method, path, body=body, headers=headers or {})
        r = c.getresponse()
        return r.status, json.loads(r.read() or b"{}")
    finally:
        c.close()


def raw_status(port, data: bytes) -> int:
    import socket
    with socket.create_connection(("127.0.0.1", port), timeout=30) as c:
        c.sendall(data)
        resp = b""
        while b"\r\n" not in resp:
            chunk = c.recv(4096)
            if not chunk:
                break
            resp += chunk
    return int(resp.split(b" ")[1])


def test_parse_generate():
    toks, mt, t = ve.parse_generate(b'{"tokens":[5,0,7],"max_tokens":9999,"temperature":-1}', 49152)
    assert toks == [5, 0, 7] and mt == 2048 and t == 0.0        # clamped as the reference (:426-429)
    toks, mt, t = ve.parse_generate(b'{"tokens":[1],"max_tokens":0,"temperature":0.5}')
    assert mt == 1 and t == 0.5
    assert ve.parse_generate(b'{"tokens":[3]}')[1] == 64         # the reference's default
    for body, msg in ((b'{"prompt":"hello"}', "tokenizer"), (b'{}', "missing"), (b'{"tokens":[]}', "non-empty"),
                      (b'{"tokens":[1.5]}', "token id"), (b'{"tokens":[49152]}', "token id"),
                      (b'{"tokens":[1],"max_tokens":"x"}', "max_tokens"), (b'[1,2]', ""), (b'{"tokens":[1', "")):
        with pytest.raises(ValueError, match=msg):
            ve.parse_generate(body, 49152)


def test_routes_without_engine():
    with ve.Server() as s:
        st, j = request(s.port, "GET", "/health")
        assert st == 200 and j["status"] == "ok" and j["engines"] == 0
        assert request(s.port, "GET", "/metrics")[0] == 200
        assert request(s.port, "POST", "/generate", b'{"tokens":[1]}')[0] == 503
        assert request(s.port, "GET", "/generate")[0] == 405
        assert request(s.port, "POST", "/health")[0] == 405
        assert request(s.port, "GET", "/nope")[0] == 404
        assert request(s.port, "GET", "/health?x=1")[0] == 200       # query strings are ignored
        assert raw_status(s.port, b"POST /generate HTTP/1.1\r\nContent-Length: 2000000\r\n\r\n" +
                          b"1" * 65536) == 413                       # over 1 MiB: answered early
        assert raw_status(s.port, b"GARBAGE\r\n\r\n") == 400
        st, j = request(s.port, "POST", "/generate", b'{"tokens":[1]}', {"Transfer-Encoding": "chunked"})
        assert st == 400 and "chunked" in j["error"]


@pytest.mark.gpu
def test_generate_over_http_matches_oracle(tmp_path):
    spec = dict(vocab=4096, hidden=576, inter=1536, layers=3, heads=9, kv_heads=3, max_pos=512)
    d = ve.synth_model(str(tmp_path / "m"), seed=21, **spec)
    p = ve.prompt(5, spec["vocab"], 10)
    with ve.Server(d, devices=[0], max_len=128) as s:
        st, j = request(s.port, "POST", "/generate", json.dumps({"tokens": p.tolist(), "max_tokens": 24}).encode())
        assert st == 200, j
        st, h = request(s.port, "GET", "/health")
        st2, m = request(s.port, "GET", "/metrics")
        bad = request(s.port, "POST", "/generate", b'{"prompt":"text"}')
    oracle.set_threads(os.cpu_count() or 1)
    want, margins = oracle.Model(d).generate(p, 24)
    assert j["tokens"] == [int(x) for x in want] and j["generated_tokens"] == 24 and j["prompt_tokens"] == 10
    assert not j["hit_stop"] and j["ms_per_token"] > 0
    assert h["engines"] == 1 and h["layers"] == 3 and h["vocab_size"] == 4096
    assert st2 == 200 and m["requests_served"] == 1 and m["tokens_per_sec"] > 0
    assert bad[0] == 400
