"""Multi-session target over the shared-memory transport: sessions are independent and match single-session runs."""

from __future__ import annotations

import threading

import torch

from conftest import mod

PAGE = 4


def _weights():
    llama = mod("models.llama")
    return (llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32),
            llama.random_weights(llama.get_config("tiny-target"), seed=2, dtype=torch.float32))


def _generate(dw, client, prompt, *, drafter_pool=None, engine=None):
    engine_mod = mod("runtime.engine")
    drafter = mod("runtime.drafter")
    edge = mod("serving.edge")
    de = engine or engine_mod.LlamaEngine(dw, num_pages=512, page_size=PAGE, max_positions=512)
    dr = drafter.DrafterRuntime(de, page_pool=drafter_pool)
    cfg = edge.DistributedAtlasConfig(k=2, d=2, max_new_tokens=10, validate_state_alignment=True)
    return edge.PagedDistributedAtlasGenerator(config=cfg, drafter=dr, target_client=client).generate(prompt)


def test_two_sessions_over_shm_match_single_session(tmp_path):
    engine_mod = mod("runtime.engine")
    target = mod("runtime.target")
    rpc = mod("serving.rpc")
    sess = mod("serving.sessions")
    native = mod("ops._native")
    dw, tw = _weights()
    prompts = [list(range(10, 40)), list(range(300, 322))]
    # Reference: each prompt alone with an in-process single-session target.
    want = []
    for p in prompts:
        te = engine_mod.LlamaEngine(tw, num_pages=512, page_size=PAGE, max_positions=512)
        want.append(_generate(dw, rpc.InProcessTargetClient(target.TargetVerifier(te, k=2, d=2)), p))

    te = engine_mod.LlamaEngine(tw, num_pages=512, page_size=PAGE, max_positions=512)
    pool = native.host().PagePool(te.num_pages - 1, PAGE)
    app = sess.MultiSessionTargetApp(lambda sid: target.TargetVerifier(te, k=2, d=2, page_pool=pool))
    base = str(tmp_path / "chan")
    server_box: dict = {}

    def server():
        ch = sess.ShmChannel(base, server=True, timeout_s=60)
        server_box["served"] = sess.serve_target_shm(app, ch)
        ch.close()

    th = threading.Thread(target=server, daemon=True)
    th.start()
    ch = sess.ShmChannel(base, server=False, timeout_s=60)
    lock = threading.Lock()
    clients = [sess.ShmTargetClient(ch, session_id=f"s{i}", lock=lock) for i in range(2)]
    de = engine_mod.LlamaEngine(dw, num_pages=512, page_size=PAGE, max_positions=512)
    dpool = native.host().PagePool(de.num_pages - 1, PAGE)
    got = [None, None]

    def run(i):
        got[i] = _generate(dw, clients[i], prompts[i], drafter_pool=dpool, engine=de)

    workers = [threading.Thread(target=run, args=(i,)) for i in range(2)]
    for w in workers:
        w.start()
    for w in workers:
        w.join(timeout=300)
    assert clients[0].health()["sessions"] == ["s0", "s1"]
    free_before = pool.free_pages
    assert clients[0].release()["released"]
    assert pool.free_pages > free_before
    clients[0].stop_server()
    th.join(timeout=60)
    ch.close()
    for g, w in zip(got, want):
        assert g is not None
        assert g.generated_token_ids == w.generated_token_ids
        assert [r.decision for r in g.rounds] == [r.decision for r in w.rounds]
    assert server_box["served"] >= 2 * 2


def test_multi_session_http_server(tmp_path):
    import threading as th

    ts = mod("serving.target_server")
    rpc = mod("serving.rpc")
    args = ts.build_parser().parse_args(["--model", "tiny-target", "--port", "0", "--device", "cpu", "--dtype",
                                         "float32", "--page-size", "4", "--k", "2", "--d", "2", "--prefix-len", "64",
                                         "--max-new-tokens-capacity", "64", "--sessions", "3"])
    app = ts.build_multi_session_app(args)
    server = rpc.make_server(app, host="127.0.0.1", port=0)
    t = th.Thread(target=server.serve_forever, daemon=True)
    t.start()
    try:
        url = f"http://127.0.0.1:{server.server_address[1]}"
        dw, _ = _weights()
        outs = []
        for sid in ("a", "b"):
            c = rpc.RemoteTargetClient(url, timeout=60, session_id=sid)
            outs.append(_generate(dw, c, list(range(5, 25))))
        assert outs[0].generated_token_ids == outs[1].generated_token_ids
        h = rpc.RemoteTargetClient(url).health()
        assert h["sessions"] == ["a", "b"]
        assert rpc.RemoteTargetClient(url, session_id="a").release()["released"]
    finally:
        server.shutdown()
        server.server_close()
