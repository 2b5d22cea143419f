"""Tensor-parallel (+ sequence-parallel) native Llama with the filtered backward.

Per layer, rank ``p`` of a TP group of size ``P`` holds heads ``[p*nh/P, (p+1)*nh/P)`` (and the
matching KV heads), FFN columns ``[p*F/P, (p+1)*F/P)`` and vocabulary rows
``[p*V/P, (p+1)*V/P)``; embedding and RMSNorm weights are replicated (their gradients are summed
over the group after the backward).  The residual stream is row-sharded (sequence parallel).

Forward (per layer, rows of this rank ``x_p``)::

    xn  = AG(rmsnorm(x_p))               qkv = xn Wqkv_p^T, RoPE      o = attn(qkv)  (local heads)
    x2_p = x_p + RS(o Wo_p^T)            xn2 = AG(rmsnorm(x2_p))       h = swiglu(xn2 Wgu_p^T)
    x_p' = x2_p + RS(h Wd_p^T)

Head: ``xf = AG(rmsnorm(x_p))``, ``logits_p = xf Wlm_p^T``, vocabulary-parallel cross entropy
(row max / sum-exp / label logit combined with three all-reduces of ``[T]`` floats).

Filtered backward: the same chain on kept rows only.  Row-parallel backward all-gathers the
kept rows of the residual gradient (padded per rank, see
:class:`~centrifuge_b200.parallel.tensor_parallel.KeptLayout`), column-parallel backward
reduce-scatters the kept-row partial sums; GEMMs run on the ``B*S_keep`` compact rows, the
attention backward is the fused restore-Q kernel on the local heads.  Reference behaviour:
the rewriter shrinks the saved inputs of Megatron's PyNodes so that the column-parallel dX
all-reduces carry ``[B, S_keep, H]`` (node_processing.cpp:369-427, megatron_tp_benchmark.py).
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from ..config import LlamaConfig
from ..filter.state import FilterSlot, FilterState
from ..ops import fused
from ..ops import gemm as G
from ..ops.reference import rope_table
from ..parallel.tensor_parallel import KeptLayout, TPGroup
from .flat import FlatParams
from .llama import CausalLMOutput, param_specs


def shard_full_params(cfg: LlamaConfig, full: Dict[str, torch.Tensor], P: int, p: int,
                      layers=None) -> Dict[str, torch.Tensor]:
    """Slice full native parameters (``wqkv = [q; k; v]``, ``wgu = [gate; up]``) for TP rank p."""
    hd, nh, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    F, V = cfg.intermediate_size, cfg.vocab_size
    nh_l, nkv_l, F_l, V_l = nh // P, nkv // P, F // P, V // P
    out = {}
    for name, t in full.items():
        if name in ("embed", "norm") or name.endswith("ln1") or name.endswith("ln2"):
            out[name] = t
        elif name == "lm_head":
            out[name] = t[p * V_l:(p + 1) * V_l]
        elif name.endswith("wqkv"):
            q = t[p * nh_l * hd:(p + 1) * nh_l * hd]
            k0 = nh * hd
            k = t[k0 + p * nkv_l * hd:k0 + (p + 1) * nkv_l * hd]
            v0 = (nh + nkv) * hd
            v = t[v0 + p * nkv_l * hd:v0 + (p + 1) * nkv_l * hd]
            out[name] = torch.cat([q, k, v], 0)
        elif name.endswith("wo"):
            out[name] = t[:, p * nh_l * hd:(p + 1) * nh_l * hd]
        elif name.endswith("wgu"):
            out[name] = torch.cat([t[p * F_l:(p + 1) * F_l], t[F + p * F_l:F + (p + 1) * F_l]], 0)
        elif name.endswith("wd"):
            out[name] = t[:, p * F_l:(p + 1) * F_l]
    return out


def replicated_names(names):
    return [n for n in names if n in ("embed", "norm") or n.endswith("ln1") or n.endswith("ln2")]


def _gather(t: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    if (t.shape[1] * t.element_size()) % 16 == 0 and t.stride(1) == 1:
        return fused.gather_rows(t, idx)
    return t.index_select(0, idx.long())


class TPLlamaCore(torch.nn.Module):
    def __init__(self, cfg: LlamaConfig, tp_group=None, device="cuda", first: int = 0,
                 last: Optional[int] = None, has_embed: bool = True, has_head: bool = True,
                 dtype=torch.bfloat16, pad_to: int = 1):
        super().__init__()
        assert not cfg.tie_word_embeddings
        self.cfg = cfg
        self.tp = TPGroup(tp_group)
        P = self.tp.size
        assert cfg.num_attention_heads % P == 0 and cfg.num_key_value_heads % P == 0
        assert cfg.intermediate_size % P == 0 and cfg.vocab_size % P == 0
        self.first = first
        self.last = cfg.num_hidden_layers if last is None else last
        self.layer_ids = range(self.first, self.last)
        self.has_embed, self.has_head = has_embed, has_head
        self.nh, self.nkv, self.hd = cfg.num_attention_heads // P, cfg.num_key_value_heads // P, cfg.head_dim
        self.F = cfg.intermediate_size // P
        self.V = cfg.vocab_size // P
        self.vocab_start = self.tp.rank * self.V
        self.flat = FlatParams(param_specs(cfg, self.layer_ids, has_embed, has_head, tp=P), device,
                               dtype=dtype, pad_to=pad_to)
        self.device = self.flat.device
        self.scale = 1.0 / math.sqrt(self.hd)
        self._rope = rope_table(cfg.max_position_embeddings, self.hd, cfg.rope_theta, self.device)
        self._pos_cache: Dict[Tuple[int, int], torch.Tensor] = {}
        self.grad_ready_hook = None
        self._anchor = torch.zeros((), device=self.device, requires_grad=True)
        self.replicated = replicated_names(self.flat.names())
        self.pending_input_grad = None
        self.last_state = None
        # Forward collectives fused with RMSNorm / the GEMMs over NVLink (parallel/tp_fused.py).
        # The gather buffers double as saved activations until the next forward, so this is for
        # schedules with one micro-batch in flight (no pipeline interleaving).
        self.use_fused_comm = False
        # micro-batches whose fused-forward activations may be alive at once (1F1B pipeline
        # stages keep up to `pp` forwarded micro-batches before their backward): each gets its
        # own set of gather slots
        self.comm_sets = 1
        self._fwd_count = 0
        self._comm = None
        self._ce_x = None  # vocabulary-parallel loss exchange over NVLink (fused mode)

    def reduce_replicated_grads(self) -> None:
        """Sum the gradients of replicated weights (embedding, RMSNorm) over the TP group.
        Call once per optimizer step, on the gradients accumulated over the micro-batches.
        The small ones (the RMSNorm weights of every layer) travel packed in one all-reduce
        instead of one collective each; large ones are reduced in place."""
        if self.tp.size == 1:
            return
        small = [self.flat.grads[n] for n in self.replicated
                 if self.flat.grads[n].numel() <= (1 << 22)]
        for n in self.replicated:
            if self.flat.grads[n].numel() > (1 << 22):
                self.tp.all_reduce_(self.flat.grads[n])
        if small:
            packed = torch.cat([g.reshape(-1) for g in small])
            self.tp.all_reduce_(packed)
            off = 0
            for g in small:
                g.copy_(packed[off:off + g.numel()].view_as(g))
                off += g.numel()

    def replicated_ranges(self):
        return [self.flat.range_of(n) for n in self.replicated]

    def load_full_(self, full: Dict[str, torch.Tensor]) -> None:
        """Copy this rank's shards of full native parameters into the flat buffer."""
        local = shard_full_params(self.cfg, full, self.tp.size, self.tp.rank)
        for name, dst in self.flat.params.items():
            dst.copy_(local[name])

    def _pos(self, B, S):
        t = self._pos_cache.get((B, S))
        if t is None:
            t = torch.arange(S, dtype=torch.int32, device=self.device).repeat(B)
            self._pos_cache[(B, S)] = t
        return t

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids=None, hidden=None, labels=None, batch_shape=None) -> CausalLMOutput:
        B, S = input_ids.shape if input_ids is not None else batch_shape
        out = _CfTPLlamaFn.apply(self._anchor, hidden, input_ids, labels, self, B, S)
        return CausalLMOutput(token_loss=out) if self.has_head else CausalLMOutput(hidden=out)

    def _forward_impl(self, input_ids, hidden_in, labels, B, S):
        p, cfg, tp = self.flat.params, self.cfg, self.tp
        T = B * S
        P = tp.size
        assert T % P == 0
        shard = T // P
        r0 = tp.rank * shard
        nh, nkv, hd = self.nh, self.nkv, self.hd
        sv = {"B": B, "S": S, "layers": []}
        pos = self._pos(B, S)
        if self.has_embed:
            ids = input_ids.reshape(-1).contiguous()
            sv["ids_local"] = ids[r0:r0 + shard].contiguous()
            x = fused.embedding_fwd(p["embed"], sv["ids_local"])
        else:
            x = hidden_in.contiguous()
        comm = self._fused_comm(T) if (self.use_fused_comm and P > 1) else None
        if comm is not None:
            return self._forward_fused(comm, x, input_ids, labels, B, S, sv, pos)
        for i in self.layer_ids:
            pre = f"layers.{i}."
            L = {"x": x}
            xn_p, r1 = fused.rmsnorm_fwd(x, p[pre + "ln1"], cfg.rms_norm_eps)
            xn = tp.all_gather_rows(xn_p)
            # RoPE of the q and k heads runs in the projection's epilogue
            qkv = G.linear_fwd_rope(xn, p[pre + "wqkv"], pos, self._rope, (nh + nkv) * hd, hd)
            o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd, scale=self.scale)
            part = G.linear_fwd(o, p[pre + "wo"])
            x2 = tp.reduce_scatter_rows(part) + x if P > 1 else G.linear_fwd(o, p[pre + "wo"], resid=x)
            xn2_p, r2 = fused.rmsnorm_fwd(x2, p[pre + "ln2"], cfg.rms_norm_eps)
            xn2 = tp.all_gather_rows(xn2_p)
            gu, h = G.linear_fwd_swiglu(xn2, p[pre + "wgu"])  # SwiGLU in the epilogue
            x = tp.reduce_scatter_rows(G.linear_fwd(h, p[pre + "wd"])) + x2 if P > 1 else \
                G.linear_fwd(h, p[pre + "wd"], resid=x2)
            L.update(xn=xn, rstd1=r1, qkv=qkv, o=o, lse=lse, x2=x2, xn2=xn2, rstd2=r2, gu=gu, h=h)
            sv["layers"].append(L)
        if not self.has_head:
            return x, sv
        xf_p, rf = fused.rmsnorm_fwd(x, p["norm"], cfg.rms_norm_eps)
        xf = tp.all_gather_rows(xf_p)
        logits = G.linear_fwd(xf, p["lm_head"])
        return self._head_loss(logits, x, xf, rf, input_ids, labels, B, S, sv)

    def _head_loss(self, logits, x, xf, rf, input_ids, labels, B, S, sv):
        tp, P = self.tp, self.tp.size
        if labels is None:
            lab = torch.full((B, S), -100, dtype=torch.long, device=x.device)
            lab[:, :-1] = input_ids[:, 1:]
        else:
            lab = labels.to(torch.long).clone()
        lab = lab.reshape(-1).contiguous()
        if P > 1 and self.use_fused_comm and logits.is_cuda:
            # row statistics exchanged over NVLink by one kernel (parallel/tp_fused.py)
            if self._ce_x is None or self._ce_x.T < lab.numel():
                from ..parallel.tp_fused import VocabParallelCE
                self._ce_x = VocabParallelCE(tp, lab.numel(), x.device)
            loss, lse_ce = self._ce_x(logits, lab, self.vocab_start)
        elif P > 1:
            pmax, psum, ptgt = fused.ce_partial(logits, lab, self.vocab_start)
            gmax = tp.all_reduce_(pmax.clone(), torch.distributed.ReduceOp.MAX)
            tot = tp.all_reduce_(psum * torch.exp(pmax - gmax))
            tgt = tp.all_reduce_(ptgt)
            lse_ce = gmax + torch.log(tot)
            loss = torch.where(lab >= 0, lse_ce - tgt, torch.zeros_like(tgt))
        else:
            loss, lse_ce = fused.ce_fwd(logits, lab)
        sv["head"] = dict(x=x, xf=xf, rstdf=rf, logits=logits, labels=lab, lse=lse_ce)
        return loss.view(B, S)[:, :-1].contiguous(), sv

    def _slots_per_set(self) -> int:
        # xn, xn2 per layer, the final norm, two for the backward's gathers
        return 2 * len(self.layer_ids) + 3

    def _fused_comm(self, T: int):
        if self._comm is None or self._comm.T != T:
            from ..parallel.tp_fused import TPFusedComm
            self._comm = TPFusedComm(self.tp, T, self.cfg.hidden_size,
                                     self.comm_sets * self._slots_per_set(), self.device)
        return self._comm

    def _forward_fused(self, comm, x, input_ids, labels, B, S, sv, pos):
        """Forward with the sequence-parallel all-gathers fused into RMSNorm + the consuming
        GEMM and the reduce-scatters fused into the row-parallel GEMMs (parallel/tp_fused.py)."""
        p, cfg, tp = self.flat.params, self.cfg, self.tp
        nh, nkv, hd = self.nh, self.nkv, self.hd
        eps = cfg.rms_norm_eps
        # this micro-batch's slot set (its gathered rows stay valid until its backward)
        base = (self._fwd_count % self.comm_sets) * self._slots_per_set()
        self._fwd_count += 1
        sv["comm_base"] = base
        for li, i in enumerate(self.layer_ids):
            pre = f"layers.{i}."
            L = {"x": x}
            xn, r1 = comm.rmsnorm_local(x, p[pre + "ln1"], eps, base + 2 * li)
            qkv = comm.gemm_ag(xn, p[pre + "wqkv"], base + 2 * li,
                               rope=(pos, self._rope, (nh + nkv) * hd, hd))
            o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd, scale=self.scale)
            x2 = comm.gemm_rs(o, p[pre + "wo"], x)
            xn2, r2 = comm.rmsnorm_local(x2, p[pre + "ln2"], eps, base + 2 * li + 1)
            gu = comm.gemm_ag(xn2, p[pre + "wgu"], base + 2 * li + 1)
            h = fused.swiglu_fwd(gu)
            x = comm.gemm_rs(h, p[pre + "wd"], x2)
            L.update(xn=xn, rstd1=r1, qkv=qkv, o=o, lse=lse, x2=x2, xn2=xn2, rstd2=r2, gu=gu, h=h)
            sv["layers"].append(L)
        sv["fused"] = True
        if not self.has_head:
            return x, sv
        fslot = base + 2 * len(self.layer_ids)
        xf, rf = comm.rmsnorm_local(x, p["norm"], eps, fslot)
        logits = comm.gemm_ag(xf, p["lm_head"], fslot)
        return self._head_loss(logits, x, xf, rf, input_ids, labels, B, S, sv)

    # ------------------------------------------------------------------ backward
    def _backward_impl(self, sv, grad_out, state: Optional[FilterState]):
        p, g, cfg, tp = self.flat.params, self.flat.grads, self.cfg, self.tp
        B, S = sv["B"], sv["S"]
        T = B * S
        nh, nkv, hd = self.nh, self.nkv, self.hd
        lay = KeptLayout(state.rows if state is not None else None, T, tp, self.device)
        if state is not None:
            rows, Sk, pos_flat, pos2d = lay.rows, state.s_keep, state.pos_flat, state.pos
        else:
            rows, Sk, pos_flat, pos2d = None, S, self._pos(B, S), None
        Tk, H = B * Sk, cfg.hidden_size
        local = None if lay.identity else lay.local
        if sv.get("fused") and tp.size > 1:
            return self._backward_fused(sv, grad_out, state, lay, rows, Sk, pos_flat, pos2d)

        def ag(dx_p):  # padded local kept rows -> compact global kept rows
            return lay.to_compact(tp.all_gather_rows(dx_p), _gather)

        def rs(part):  # compact partial sums -> padded local kept rows (summed over the group)
            if lay.identity:
                return tp.reduce_scatter_rows(part)
            z = torch.cat([part, part.new_zeros(1, part.shape[1])], 0)
            return tp.reduce_scatter_rows(lay.to_padded(z, _gather))

        def gat(t):
            return t if rows is None else _gather(t, rows)

        if self.has_head:
            hd_ = sv["head"]
            dl = grad_out.float()
            if state is not None and dl.shape[1] == S - 1:
                dl = torch.gather(dl, 1, pos2d[:, :-1].long())
            dl = torch.cat([dl, torch.zeros(B, 1, device=dl.device, dtype=dl.dtype)], 1)
            dloss = dl.reshape(-1).contiguous()
            dlogits = fused.ce_bwd(hd_["logits"], hd_["labels"], hd_["lse"], dloss, rows,
                                   vocab_start=self.vocab_start)
            xf_k = gat(hd_["xf"])
            G.linear_wgrad(dlogits, xf_k, g["lm_head"])
            dxf_p = rs(G.linear_dgrad(dlogits, p["lm_head"]))
            del dlogits, xf_k
            dx = fused.rmsnorm_bwd(dxf_p, hd_["x"], hd_["rstdf"], p["norm"], g["norm"], x_rows=local)
        else:
            dx = grad_out.contiguous()
        for li, i in reversed(list(enumerate(self.layer_ids))):
            L = sv["layers"][li]
            pre = f"layers.{i}."
            dY = ag(dx)
            h_k = gat(L["h"])
            G.linear_wgrad(dY, h_k, g[pre + "wd"])
            dh = G.linear_dgrad(dY, p[pre + "wd"])
            del h_k, dY
            dgu = fused.swiglu_bwd(dh, L["gu"], rows)
            del dh
            xn2_k = gat(L["xn2"])
            G.linear_wgrad(dgu, xn2_k, g[pre + "wgu"])
            dxn2_p = rs(G.linear_dgrad(dgu, p[pre + "wgu"]))
            del dgu, xn2_k
            dx2 = fused.rmsnorm_bwd(dxn2_p, L["x2"], L["rstd2"], p[pre + "ln2"], g[pre + "ln2"],
                                    x_rows=local, dres=dx)
            del dxn2_p, dx
            dY2 = ag(dx2)
            o_k = gat(L["o"])
            G.linear_wgrad(dY2, o_k, g[pre + "wo"])
            do = G.linear_dgrad(dY2, p[pre + "wo"])
            del dY2
            qkv_k = gat(L["qkv"])
            lse_k = L["lse"] if rows is None else _gather(L["lse"], rows)
            dqkv = fused.attn_bwd(qkv_k, L["qkv"], o_k, do, lse_k,
                                  pos2d if pos2d is not None else pos_flat.view(B, S),
                                  B, S, Sk, nh, nkv, hd, scale=self.scale,
                                  rope_table=self._rope)  # RoPE backward in the epilogue
            del qkv_k, lse_k, o_k, do
            xn_k = gat(L["xn"])
            G.linear_wgrad(dqkv, xn_k, g[pre + "wqkv"])
            dxn_p = rs(G.linear_dgrad(dqkv, p[pre + "wqkv"]))
            del dqkv, xn_k
            dx = fused.rmsnorm_bwd(dxn_p, L["x"], L["rstd1"], p[pre + "ln1"], g[pre + "ln1"],
                                   x_rows=local, dres=dx2)
            del dxn_p, dx2
            sv["layers"][li] = None
        if self.has_embed:
            n = lay.count if not lay.identity else dx.shape[0]
            fused.embedding_bwd(dx[:n], sv["ids_local"], g["embed"],
                                id_rows=None if lay.identity else lay.local[:n])
        if self.has_embed:
            return None
        return dx


def _backward_fused_impl(self, sv, grad_out, state, lay, rows, Sk, pos_flat, pos2d):
    """Filtered backward with the all-gathers fused into the RMSNorm backward + the consuming
    dgrad GEMM and the reduce-scatters fused into the column-parallel dgrad GEMMs.  Kept rows
    stay in the compact global order: rank q's kept rows are rows [start_q, start_q + count_q)
    of every gathered tensor and of every partial sum (rank-major because shards are row
    ranges), so the GEMMs see exactly the kept rows; local rows keep the padded layout of
    :class:`KeptLayout` (C rows, zero padding)."""
    from ..parallel.tp_fused import Segments
    p, g, cfg, tp = self.flat.params, self.flat.grads, self.cfg, self.tp
    comm = self._comm
    B, S = sv["B"], sv["S"]
    nh, nkv, hd = self.nh, self.nkv, self.hd
    seg = Segments(lay.counts, self.device)
    C = lay.C
    local = None if lay.identity else lay.local
    slot_a = sv.get("comm_base", 0) + 2 * len(self.layer_ids) + 1
    slot_b = slot_a + 1

    def gat(t):
        return t if rows is None else _gather(t, rows)

    if self.has_head:
        hd_ = sv["head"]
        dl = grad_out.float()
        if state is not None and dl.shape[1] == S - 1:
            dl = torch.gather(dl, 1, pos2d[:, :-1].long())
        dl = torch.cat([dl, torch.zeros(B, 1, device=dl.device, dtype=dl.dtype)], 1)
        dloss = dl.reshape(-1).contiguous()
        dlogits = fused.ce_bwd(hd_["logits"], hd_["labels"], hd_["lse"], dloss, rows,
                               vocab_start=self.vocab_start)
        xf_k = gat(hd_["xf"])
        G.linear_wgrad(dlogits, xf_k, g["lm_head"])
        dxf_p = comm.gemm_rs(dlogits, p["lm_head"], None, seg=seg, b_mn=True, out_rows=C)
        del dlogits, xf_k
        # dx of the final norm; its kept rows are all-gathered by the last layer's down dgrad
        dx = fused.rmsnorm_bwd(dxf_p, hd_["x"], hd_["rstdf"], p["norm"], g["norm"], x_rows=local)
    else:
        # a pipeline stage below the head: the gradient of its output, this rank's kept rows
        # (padded local layout, as this function returns it)
        dx = grad_out.contiguous()
    layers = list(enumerate(self.layer_ids))
    dYg = comm.place_rows(dx, slot_a, seg)
    for li, i in reversed(layers):
        L = sv["layers"][li]
        pre = f"layers.{i}."
        # ---- MLP: dgrad first (it gathers the rows), then wgrad reads the gathered rows
        dh = comm.gemm_ag(dYg, p[pre + "wd"], slot_a, seg=seg, b_mn=True)
        h_k = gat(L["h"])
        G.linear_wgrad(dYg, h_k, g[pre + "wd"])
        del h_k
        dgu = fused.swiglu_bwd(dh, L["gu"], rows)
        del dh
        xn2_k = gat(L["xn2"])
        G.linear_wgrad(dgu, xn2_k, g[pre + "wgu"])
        dxn2_p = comm.gemm_rs(dgu, p[pre + "wgu"], None, seg=seg, b_mn=True, out_rows=C)
        del dgu, xn2_k
        dx2 = fused.rmsnorm_bwd(dxn2_p, L["x2"], L["rstd2"], p[pre + "ln2"], g[pre + "ln2"],
                                x_rows=local, dres=dx)
        dY2g = comm.place_rows(dx2, slot_b, seg)
        del dxn2_p, dx
        # ---- attention
        do = comm.gemm_ag(dY2g, p[pre + "wo"], slot_b, seg=seg, b_mn=True)
        o_k = gat(L["o"])
        G.linear_wgrad(dY2g, o_k, g[pre + "wo"])
        qkv_k = gat(L["qkv"])
        lse_k = L["lse"] if rows is None else _gather(L["lse"], rows)
        dqkv = fused.attn_bwd(qkv_k, L["qkv"], o_k, do, lse_k,
                              pos2d if pos2d is not None else pos_flat.view(B, S),
                              B, S, Sk, nh, nkv, hd, scale=self.scale, rope_table=self._rope)
        del qkv_k, lse_k, o_k, do
        xn_k = gat(L["xn"])
        G.linear_wgrad(dqkv, xn_k, g[pre + "wqkv"])
        dxn_p = comm.gemm_rs(dqkv, p[pre + "wqkv"], None, seg=seg, b_mn=True, out_rows=C)
        del dqkv, xn_k
        dx = fused.rmsnorm_bwd(dxn_p, L["x"], L["rstd1"], p[pre + "ln1"], g[pre + "ln1"],
                               x_rows=local, dres=dx2)
        if li > 0:
            dYg = comm.place_rows(dx, slot_a, seg)
        del dxn_p, dx2
        sv["layers"][li] = None
    if self.has_embed:
        n = lay.count if not lay.identity else dx.shape[0]
        fused.embedding_bwd(dx[:n], sv["ids_local"], g["embed"],
                            id_rows=None if lay.identity else lay.local[:n])
        return None
    return dx


TPLlamaCore._backward_fused = _backward_fused_impl


class _CfTPLlamaFn(torch.autograd.Function):
    """Autograd node of a TP native Llama stage (``_Cf`` prefix: the rewriter attaches the mask)."""

    @staticmethod
    def forward(ctx, anchor, hidden, input_ids, labels, model: TPLlamaCore, B: int, S: int):
        out, sv = model._forward_impl(input_ids, hidden, labels, B, S)
        ctx.model, ctx.saved, ctx.slot = model, sv, FilterSlot()
        ctx.hidden_in = not model.has_embed
        return out

    @staticmethod
    def backward(ctx, grad_out):
        sv, ctx.saved = ctx.saved, None
        dx = ctx.model._backward_impl(sv, grad_out, ctx.slot.state)
        if ctx.hidden_in:
            # the input gradient is in the kept-row layout of the pipeline, not the input's
            # shape: hand it to the pipeline schedule instead of autograd
            ctx.model.pending_input_grad = dx
        ctx.model.last_state = ctx.slot.state
        return None, None, None, None, None, None, None

    @staticmethod
    def cf_attach(ctx, mask):
        ctx.slot.attach(mask)
