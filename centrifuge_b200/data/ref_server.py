"""Reference-loss service: per-token loss of a reference model, served over TCP.

Reference: ref_server.py and model/utils.py:75-215.  Wire format (kept for interoperability):
a 4-byte big-endian length followed by a pickle payload.  Requests are
``List[List[int]]`` (token ids per sample); replies are ``{"loss": List[List[float]]}`` with
``len(ids) - 1`` per-token CE losses per sample.

* :func:`obtain_ref_loss` -- per-token CE of a causal LM (HF or native model) on a batch of
  token-id lists (right-aligned / left-padded as in the reference).
* :class:`NGramModel` -- bigram / trigram negative log-probabilities from count tables
  (model/n_gram.py), without the NLTK dependency.
* :class:`RefLossServer` -- accepts ``num_connects`` clients, one reader thread per client
  feeding one model loop that answers each client in order.
* :func:`init_single_socket` / :func:`init_multiple_sockets` / :func:`init_socket` -- client
  side: a connected socket plus send/receive worker threads and queues.
* :class:`VllmClient` -- reference loss from a vLLM OpenAI-compatible server (prompt logprobs).
"""
from __future__ import annotations

import json
import math
import os
import pickle
import queue
import socket
import struct
import threading
from typing import Callable, List, Optional, Sequence, Tuple

import torch


# ------------------------------------------------------------------ framing
def send_all(sock: socket.socket, payload: bytes) -> None:
    sock.sendall(struct.pack(">I", len(payload)) + payload)


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        part = sock.recv(min(1 << 16, n - len(buf)))
        if not part:
            raise ConnectionError("peer closed the connection")
        buf += part
    return bytes(buf)


def receive_all(sock: socket.socket) -> bytes:
    (n,) = struct.unpack(">I", _recv_exact(sock, 4))
    return _recv_exact(sock, n)


# ------------------------------------------------------------------ reference losses
@torch.inference_mode()
def obtain_ref_loss(model, messages: Sequence[Sequence[int]], pad_id: int = 0,
                    device=None, return_pickle: bool = False):
    """Per-token CE losses (``len(m) - 1`` values per message) of a causal LM.

    Messages of different lengths are left-padded to a common length, as the reference does.
    ``model(input_ids)`` may return an object with ``.logits`` or the logits tensor.
    """
    sizes = [len(m) for m in messages]
    L = max(sizes)
    ids = torch.tensor([[pad_id] * (L - len(m)) + list(m) for m in messages], dtype=torch.long)
    if device is None:
        device = next(model.parameters()).device if hasattr(model, "parameters") else "cpu"
    out = model(ids.to(device))
    logits = out.logits if hasattr(out, "logits") else out
    lf = logits[:, :-1].float()
    loss = torch.nn.functional.cross_entropy(lf.reshape(-1, lf.shape[-1]),
                                             ids[:, 1:].reshape(-1).to(lf.device),
                                             reduction="none").view(len(messages), L - 1)
    rows = loss.cpu().tolist()
    res = [rows[i][L - sizes[i]:] for i in range(len(messages))]
    return pickle.dumps({"loss": res}) if return_pickle else res


@torch.inference_mode()
def obtain_ref_loss_cross_tokenizer(model, tokenizer, target_input_ids: Sequence[Sequence[int]],
                                    target_tokenizer, device=None, tokenize_args=None,
                                    return_pickle: bool = False):
    """Reference losses for target-tokenized messages when the reference model has its own
    tokenizer (model/utils.py:76-106 with ``manuel_matching``): decode the target ids, tokenize
    the text with the reference tokenizer, compute the reference model's per-token losses and
    move them onto the target tokens (:func:`centrifuge_b200.data.align.align_ref_target_tokens`).
    Returns ``len(m) - 1`` losses per target message."""
    from .align import align_ref_target_tokens, tokenized_prompts
    strip_bos = bool(getattr(target_tokenizer, "add_bos_token", False))
    texts = target_tokenizer.batch_decode([list(m)[1:] if strip_bos else list(m)
                                           for m in target_input_ids])
    ref_ids = [list(x) for x in tokenizer(texts, **(tokenize_args or {}))["input_ids"]]
    pad = getattr(tokenizer, "pad_token_id", None)
    losses = obtain_ref_loss(model, ref_ids, pad_id=0 if pad is None else pad, device=device)
    aligned = align_ref_target_tokens(tokenized_prompts(tokenizer, ref_ids),
                                      tokenized_prompts(target_tokenizer, target_input_ids),
                                      losses)
    return pickle.dumps({"loss": aligned}) if return_pickle else aligned


class NGramModel:
    """Bigram / trigram reference loss from count tables.

    ``word1_num.json``, ``word2_num.json``, ``word3_num.json`` map ``str(token)``,
    ``str((t1, t2))`` and ``str((t1, t2, t3))`` (lower-cased tokens) to counts.  A missing
    n-gram gets probability 1e-20 (model/n_gram.py:25-57).
    """

    def __init__(self, n_gram_path: str, tokenizer=None):
        def load(name):
            with open(os.path.join(n_gram_path, name)) as f:
                return json.load(f)
        self.f1, self.f2, self.f3 = load("word1_num.json"), load("word2_num.json"), load("word3_num.json")
        self.tokenizer = tokenizer

    def _probs(self, tokens: List[str], n: int) -> List[float]:
        tokens = [t.lower() for t in tokens]
        out = []
        for i in range(len(tokens) - n + 1):
            gram = tuple(tokens[i:i + n])
            num = (self.f2 if n == 2 else self.f3).get(str(gram), 0)
            ctx = gram[0] if n == 2 else gram[:2]
            den = (self.f1 if n == 2 else self.f2).get(str(ctx), 0)
            p = 1e-20 if num == 0 else num / den
            out.append(-math.log(p))
        return out

    def bigram_loss(self, tokens: List[str]) -> List[float]:
        return self._probs(tokens, 2)

    def trigram_loss(self, tokens: List[str]) -> List[float]:
        return self._probs(tokens, 3)

    def obtain_ngram_loss(self, messages, model: str = "bigram", return_pickle: bool = False):
        toks = [self.tokenizer.convert_ids_to_tokens(m) if self.tokenizer else [str(t) for t in m]
                for m in messages]
        fn = self.bigram_loss if model == "bigram" else self.trigram_loss
        res = [fn(t) for t in toks]
        return pickle.dumps({"loss": res}) if return_pickle else res


class VllmClient:
    """Reference loss from a vLLM server's prompt logprobs (data/build_data.py:209-231)."""

    def __init__(self, url: str):
        import requests
        self.url = url.rstrip("/")
        self.session = requests.Session()
        r = self.session.get(self.url + "/v1/models", timeout=30)
        self.model = r.json()["data"][0]["id"]

    def get_ref_loss(self, prompts: List[str]) -> List[List[float]]:
        r = self.session.post(self.url + "/v1/completions", json=dict(
            model=self.model, prompt=prompts, echo=True, n=1, max_tokens=1, logprobs=1),
            timeout=600)
        return [[-x for x in c["logprobs"]["token_logprobs"][1:-1]] for c in r.json()["choices"]]


# ------------------------------------------------------------------ server
class RefLossServer:
    """TCP server answering reference-loss requests from ``num_connects`` clients."""

    def __init__(self, loss_fn: Callable[[List[List[int]]], List[List[float]]],
                 host: str = "0.0.0.0", port: int = 65432, num_connects: int = 1):
        self.loss_fn = loss_fn
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.sock.bind((host, port))
        self.sock.listen(max(1, num_connects))
        self.port = self.sock.getsockname()[1]
        self.num_connects = num_connects
        self.requests: "queue.Queue" = queue.Queue()
        self.clients: List[socket.socket] = []
        self.served = 0
        self._stop = threading.Event()

    def _reader(self, cid: int, conn: socket.socket):
        try:
            while not self._stop.is_set():
                msg = pickle.loads(receive_all(conn))
                if not msg:  # an empty request closes the client
                    break
                self.requests.put((cid, msg))
        except (ConnectionError, OSError, EOFError):
            pass
        self.requests.put((cid, None))

    def serve_forever(self, max_requests: Optional[int] = None) -> None:
        while len(self.clients) < self.num_connects:
            conn, _ = self.sock.accept()
            self.clients.append(conn)
            threading.Thread(target=self._reader, args=(len(self.clients) - 1, conn),
                             daemon=True).start()
        open_clients = len(self.clients)
        while open_clients > 0 and not self._stop.is_set():
            cid, msg = self.requests.get()
            if msg is None:
                open_clients -= 1
                continue
            send_all(self.clients[cid], pickle.dumps({"loss": self.loss_fn(msg)}))
            self.served += 1
            if max_requests is not None and self.served >= max_requests:
                break
        self.close()

    def close(self) -> None:
        self._stop.set()
        for c in self.clients:
            try:
                c.close()
            except OSError:
                pass
        self.sock.close()


# ------------------------------------------------------------------ client
def init_single_socket(host: str, port: int) -> Tuple["queue.Queue", "queue.Queue"]:
    """Connect; returns ``(recv_queue, send_queue)`` served by two worker threads."""
    sock = socket.create_connection((host, int(port)))
    recv_q: "queue.Queue" = queue.Queue()
    send_q: "queue.Queue" = queue.Queue()

    def sender():
        while True:
            msg = send_q.get()
            try:
                send_all(sock, pickle.dumps(msg))
            except OSError:
                break
            if not msg:
                break

    def receiver():
        while True:
            try:
                recv_q.put(pickle.loads(receive_all(sock)))
            except (ConnectionError, OSError, EOFError):
                break

    threading.Thread(target=sender, daemon=True).start()
    threading.Thread(target=receiver, daemon=True).start()
    return recv_q, send_q


def init_multiple_sockets(hosts: str, ports: str):
    """``hosts="h1@h2"``, ``ports="p1,p2@p3"`` -> one queue pair per (host, port)."""
    hs = hosts.split("@")
    ps = [p.split(",") for p in ports.split("@")]
    assert len(hs) == len(ps), "Invalid hosts:ports configuration."
    return [init_single_socket(h, p) for h, plist in zip(hs, ps) for p in plist]


def init_socket(args, selected_host: Optional[int] = None):
    hosts = args.ref_socket_hosts.split(",")
    ports = args.ref_socket_ports.split(",")
    assert len(hosts) == 1 or len(hosts) == len(ports), "Invalid hosts:ports configuration."
    if selected_host is None:
        import torch.distributed as dist
        selected_host = dist.get_rank() % len(ports) if dist.is_initialized() else 0
    host = hosts[selected_host] if len(hosts) > 1 else hosts[0]
    return init_single_socket(host, int(ports[selected_host]))


def main():
    import argparse
    ap = argparse.ArgumentParser(description="reference-loss server")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=65432)
    ap.add_argument("--num_connects", type=int, default=4)
    ap.add_argument("--model_type", choices=("llm", "bigram", "trigram"), default="llm")
    ap.add_argument("--model_name", default="TinyLlama/TinyLlama_v1.1")
    ap.add_argument("--target_tokenizer", default=None)
    ap.add_argument("--context_length", type=int, default=2048)
    a = ap.parse_args()
    if a.model_type == "llm":
        from transformers import AutoModelForCausalLM
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        model = AutoModelForCausalLM.from_pretrained(a.model_name, torch_dtype=torch.bfloat16).to(dev).eval()
        fn = lambda msgs: obtain_ref_loss(model, msgs)  # noqa: E731
    else:
        from transformers import AutoTokenizer
        ng = NGramModel(a.model_name, AutoTokenizer.from_pretrained(a.target_tokenizer or "TinyLlama/TinyLlama_v1.1"))
        fn = lambda msgs: ng.obtain_ngram_loss(msgs, a.model_type)  # noqa: E731
    srv = RefLossServer(fn, a.host, a.port, a.num_connects)
    print(f"reference-loss server listening on {a.host}:{srv.port}", flush=True)
    srv.serve_forever()


if __name__ == "__main__":
    main()
