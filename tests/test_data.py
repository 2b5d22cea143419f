"""Data pipeline pieces: packing, collation, cache naming, reference-loss service."""
import json
import threading

import torch

from centrifuge_b200.arguments import get_cache_dir, parse_args
from centrifuge_b200.data.build_data import collate_fn, pack_token_ids
from centrifuge_b200.data.ref_server import (NGramModel, RefLossServer, init_single_socket,
                                             obtain_ref_loss)
from centrifuge_b200.data.synthetic import SyntheticTokenData


def test_pack_token_ids():
    seqs = [[1, 2, 3], [4, 5, 6, 7, 8], [9], [10, 11]]
    rows, lengths, smap = pack_token_ids(seqs, 4)
    assert rows == [[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11]]
    assert lengths == [4, 4, 3] and sum(lengths) == 11


def test_collate_left_pads():
    b = collate_fn([{"input_ids": [5, 6, 7], "ref_loss": [0.1, 0.2], "length": 3},
                    {"input_ids": [8], "ref_loss": [], "length": 1}])
    assert b["input_ids"].tolist() == [[5, 6, 7], [0, 0, 8]]
    assert b["attention_mask"].tolist() == [[1, 1, 1], [0, 0, 1]]
    assert b["length"] == [3, 1] and b["ref_loss"][1] == []


def test_cache_dir_ignores_non_identifying_args(tmp_path, monkeypatch):
    monkeypatch.setenv("HF_HOME", str(tmp_path))
    a = parse_args(["--output_dir", "x", "--learning_rate", "1e-4"])
    b = parse_args(["--output_dir", "x", "--learning_rate", "1e-4", "--ref_socket_hosts", "h"])
    c = parse_args(["--output_dir", "x", "--learning_rate", "2e-4"])
    da, db, dc = get_cache_dir(a)[0], get_cache_dir(b)[0], get_cache_dir(c)[0]
    assert da == db and da != dc


def test_synthetic_data_distribution():
    d = SyntheticTokenData(100, 4, 64, seed=1, pin=False)
    b = d.sample()
    assert b.input_ids.shape == (4, 64) and b.ref_loss.shape == (4, 63)
    assert 1.0 < torch.log(b.ref_loss).mean().item() + 0.3 and b.ref_loss.min() > 0


def test_ref_loss_server_roundtrip():
    fn = lambda msgs: [[float(len(m))] * (len(m) - 1) for m in msgs]  # noqa: E731
    srv = RefLossServer(fn, "127.0.0.1", 0, num_connects=1)
    th = threading.Thread(target=srv.serve_forever, kwargs={"max_requests": 2}, daemon=True)
    th.start()
    recv_q, send_q = init_single_socket("127.0.0.1", srv.port)
    send_q.put([[1, 2, 3], [4, 5]])
    send_q.put([[7, 8, 9, 10]])
    assert recv_q.get(timeout=10)["loss"] == [[3.0, 3.0], [2.0]]
    assert recv_q.get(timeout=10)["loss"] == [[4.0, 4.0, 4.0]]
    th.join(timeout=10)


def test_obtain_ref_loss_matches_ce():
    torch.manual_seed(0)
    emb = torch.nn.Embedding(20, 20)
    model = lambda ids: emb(ids)  # noqa: E731 - logits = embedding rows
    msgs = [[1, 2, 3, 4], [5, 6]]
    out = obtain_ref_loss(model, msgs, device="cpu")
    lg = emb(torch.tensor([[1, 2, 3, 4]]))
    want = torch.nn.functional.cross_entropy(lg[0, :-1], torch.tensor([2, 3, 4]), reduction="none")
    assert torch.allclose(torch.tensor(out[0]), want.detach(), atol=1e-5) and len(out[1]) == 1


def test_ngram_model(tmp_path):
    (tmp_path / "word1_num.json").write_text(json.dumps({"a": 4, "b": 2}))
    (tmp_path / "word2_num.json").write_text(json.dumps({str(("a", "b")): 2, str(("b", "a")): 1}))
    (tmp_path / "word3_num.json").write_text(json.dumps({str(("a", "b", "a")): 1}))
    ng = NGramModel(str(tmp_path))
    bi = ng.bigram_loss(["A", "b", "a"])
    assert abs(bi[0] - (-torch.log(torch.tensor(0.5)).item())) < 1e-6
    tri = ng.trigram_loss(["a", "b", "a"])
    assert abs(tri[0] - (-torch.log(torch.tensor(0.5)).item())) < 1e-6
