"""Gated DeltaNet layer on the libgdn_b200 kernels.

Prefill (T tokens), five launches of the library's kernels:
    x [B,T,D] -> RMSNorm
              -> q,k = L2norm(SiLU(conv4(x Wq^T))), v = SiLU(conv4(x Wv^T)), z = x Wz^T and
                 [a | b] = x [Wa | Wb]^T, one persistent tcgen05 GEMM launch over the five segments
              -> chunked gated delta rule (grouped value heads, [B,T,H,D] layout; a and b read
                 in place from the [B,T,2Hv] projection output as token rows)
              -> gated RMSNorm(o) * SiLU(z) -> y Wo^T (the same GEMM kernel, one plain segment)
Decode (1 token) runs the same blocks with the carried recurrent state
[B,Hv,dk,dv] fp32 and the three conv histories [B,C,3] bf16 (the last three
projected values per channel); ``prefill`` returns both so decode continues a
prefilled sequence.  The decode projections are one weight-streaming GEMV
launch over that history (no recompute of the last four tokens).

Composition follows the reference layer (gdn_layer.py:120-199) with the
additions of the BASELINE layer (L2-normalised q/k, 16 q/k heads shared by 32
value heads, z-gated output norm, per-head A_log/dt_bias); weights are
synthetic N(0, 0.02) (config 3).  No transposes are materialised between
kernels: projections write [B,T,H*D], which the prefill reads as [B,T,H,D].
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, ops


@dataclass
class GDNConfig:
    hidden: int = 2048
    n_qk: int = 16          # q/k heads
    n_v: int = 32           # value heads
    dk: int = 128
    dv: int = 128
    conv: int = 4
    eps: float = 1e-6

    @property
    def qk_dim(self):
        return self.n_qk * self.dk

    @property
    def v_dim(self):
        return self.n_v * self.dv


def make_weights(cfg: GDNConfig, device="cuda", seed=0, std=0.02):
    """Random weights of config 3 (bf16 ~N(0, std)); A_log / dt_bias follow the
    BASELINE gate distribution (log-decay = -0.1 * softplus(a))."""
    g = torch.Generator(device=device).manual_seed(seed)

    def w(*shape, s=std):
        return (torch.randn(*shape, generator=g, device=device) * s).bfloat16()

    D = cfg.hidden
    return dict(
        norm_gamma=torch.ones(D, dtype=torch.bfloat16, device=device),
        W_q=w(cfg.qk_dim, D), conv_q=w(cfg.qk_dim, cfg.conv, s=0.5),
        W_k=w(cfg.qk_dim, D), conv_k=w(cfg.qk_dim, cfg.conv, s=0.5),
        W_v=w(cfg.v_dim, D), conv_v=w(cfg.v_dim, cfg.conv, s=0.5),
        W_z=w(cfg.v_dim, D),
        W_ab=w(2 * cfg.n_v, D),
        A_log=torch.full((cfg.n_v,), math.log(0.1), device=device),
        dt_bias=torch.zeros(cfg.n_v, device=device),
        onorm_gamma=torch.ones(cfg.dv, dtype=torch.bfloat16, device=device),
        W_o=w(D, cfg.v_dim),
    )


class GDNLayer:
    """B200 Gated DeltaNet layer; every op is a libgdn_b200 kernel."""

    def __init__(self, weights: dict, cfg: GDNConfig | None = None):
        self.w = weights
        self.cfg = cfg or GDNConfig()
        self.scale = self.cfg.dk ** -0.5
        # the a | b gate rows padded with zero rows to the projection kernel's 128-channel tile
        W_ab = weights["W_ab"]
        pad = (-W_ab.shape[0]) % 128
        self.W_ab_tile = torch.cat([W_ab, W_ab.new_zeros(pad, W_ab.shape[1])]) if pad else W_ab

    def init_state(self, B: int, device="cuda", fill=torch.zeros):
        """Zero state (``fill=torch.empty``: buffers a prefill overwrites completely)."""
        c = self.cfg
        return dict(
            recurrent=fill(B, c.n_v, c.dk, c.dv, dtype=torch.float32, device=device),
            conv_q=fill(B, c.qk_dim, c.conv - 1, dtype=torch.bfloat16, device=device),
            conv_k=fill(B, c.qk_dim, c.conv - 1, dtype=torch.bfloat16, device=device),
            conv_v=fill(B, c.v_dim, c.conv - 1, dtype=torch.bfloat16, device=device),
        )

    def _project(self, xn, state_in, state_out):
        """q, k (L2-normalised per head), v, z and the a|b gate logits [B,T,128] for
        xn [B,T,D], all in one launch."""
        c, w = self.cfg, self.w
        si = state_in or {}
        # q | k | v (conv4 + SiLU, q/k L2-normalised per head), z, a | b (plain rows)
        q, k, v, z, ab = ops.proj_multi(xn, [
            dict(W=w["W_q"], conv_w=w["conv_q"], l2norm_group=c.dk, conv_state_in=si.get("conv_q"),
                 conv_state_out=state_out["conv_q"]),
            dict(W=w["W_k"], conv_w=w["conv_k"], l2norm_group=c.dk, conv_state_in=si.get("conv_k"),
                 conv_state_out=state_out["conv_k"]),
            dict(W=w["W_v"], conv_w=w["conv_v"], conv_state_in=si.get("conv_v"), conv_state_out=state_out["conv_v"]),
            dict(W=w["W_z"]),
            dict(W=self.W_ab_tile),
        ])
        return q, k, v, z, ab

    @torch.no_grad()
    def prefill(self, x: torch.Tensor, state: dict | None = None, trace: dict | None = None):
        """x [B,T,D] bf16 -> (y [B,T,D] bf16, state after the last token).
        ``trace``: a dict that receives the intermediate tensors (xn, q, k, v, z,
        a, b [B,Hv,T], o [B,T,Hv,dv], y_norm) for stage-by-stage checks."""
        c, w = self.cfg, self.w
        B, T, D = x.shape
        xn = ops.rmsnorm(x.reshape(B * T, D), w["norm_gamma"], c.eps).reshape(B, T, D)
        new_state = self.init_state(B, x.device, fill=torch.empty)   # written by the projections and prefill
        q, k, v, z, ab = self._project(xn, state, new_state)
        a, b = ab[..., :c.n_v], ab[..., c.n_v:2 * c.n_v]          # [B, T, Hv] token rows, read in place
        o, S = ops.prefill(q.view(B, T, c.n_qk, c.dk), k.view(B, T, c.n_qk, c.dk), v.view(B, T, c.n_v, c.dv),
                           w["A_log"], a, b, dt_bias=w["dt_bias"],
                           state_in=None if state is None else state["recurrent"],
                           scale=self.scale, layout="bthd", state_out=new_state["recurrent"], gates="bth")
        y = ops.gated_rmsnorm(o.view(B * T * c.n_v, c.dv), z.view(B * T * c.n_v, c.dv), w["onorm_gamma"], c.eps)
        (out,) = ops.proj_multi(y.view(B, T, c.v_dim), [dict(W=w["W_o"])])
        if trace is not None:
            trace.update(xn=xn, q=q, k=k, v=v, z=z, a=a.transpose(1, 2), b=b.transpose(1, 2), o=o,
                         y_norm=y.view(B, T, c.v_dim))
        return out, new_state

    @torch.no_grad()
    def decode(self, x: torch.Tensor, state: dict, out_state: dict | None = None):
        """One token: x [B,1,D] bf16 -> (y [B,1,D] bf16, state).  The recurrent
        state is updated in place; conv histories go to ``out_state`` (fresh
        buffers by default; ``out_state=state`` updates them in place too).

        Three launches: RMSNorm + q|k|v (conv4, SiLU) + z + a + b as one
        weight-streaming GEMV over the cached conv history (gdn_decode_proj_fwd),
        the recurrence step with the q/k L2 norm and the gated output norm folded
        in (gdn_decode_step_gated; the GEMV needs no cross-CTA reduction and the
        output projection reads y directly), and the output projection (the same
        GEMV kernel).  All shapes are static, so the call can be captured in a
        CUDA graph."""
        c, w = self.cfg, self.w
        B = x.shape[0]
        D = c.hidden
        if out_state is None:
            out_state = dict(recurrent=state["recurrent"],
                             conv_q=torch.empty_like(state["conv_q"]), conv_k=torch.empty_like(state["conv_k"]),
                             conv_v=torch.empty_like(state["conv_v"]))
        q, k, v, z, a, b = ops.decode_proj(x.reshape(B, D), [
            dict(W=w["W_q"], conv_w=w["conv_q"], conv_state_in=state["conv_q"], conv_state_out=out_state["conv_q"]),
            dict(W=w["W_k"], conv_w=w["conv_k"], conv_state_in=state["conv_k"], conv_state_out=out_state["conv_k"]),
            dict(W=w["W_v"], conv_w=w["conv_v"], conv_state_in=state["conv_v"], conv_state_out=out_state["conv_v"]),
            dict(W=w["W_z"]),
            dict(W=w["W_ab"][:c.n_v]),
            dict(W=w["W_ab"][c.n_v:]),
        ], norm_gamma=w["norm_gamma"], eps=c.eps)
        y = ops.decode_step_gated(q.view(B, c.n_qk, c.dk), k.view(B, c.n_qk, c.dk), v.view(B, c.n_v, c.dv), a, b,
                                  w["A_log"], w["dt_bias"], state["recurrent"], z.view(B, c.n_v, c.dv),
                                  w["onorm_gamma"], c.eps, scale=self.scale, state_out=out_state["recurrent"],
                                  l2norm_qk=True)
        (out,) = ops.decode_proj(y.view(B, c.v_dim), [dict(W=w["W_o"])])
        return out.view(B, 1, D), out_state


class DecodeGraph:
    """A CUDA graph of one ``GDNLayer.decode`` step over static buffers, so a
    decode loop costs one graph launch per token.  The recurrent state and the
    conv histories of ``state`` are updated in place by every step."""

    def __init__(self, layer: GDNLayer, state: dict, B: int, overlap: bool = True):
        """``overlap``: capture the step's kernels with programmatic dependent
        launch (gdn_set_launch_overlap), so each launches while its predecessor
        finishes and the projections stream their weights early."""
        self.layer = layer
        dev = state["recurrent"].device
        self.x = torch.zeros(B, 1, layer.cfg.hidden, dtype=torch.bfloat16, device=dev)
        self.state = state
        # warm up once outside the graph (first-call set-up of the kernels) on scratch copies
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            scratch = {k_: v_.clone() for k_, v_ in state.items()}
            layer.decode(self.x, scratch, scratch)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        lib = _lib.lib()
        lib.gdn_set_launch_overlap(1 if overlap else 0)
        try:
            with torch.cuda.graph(self.graph):
                self.y, _ = layer.decode(self.x, state, state)
        finally:
            lib.gdn_set_launch_overlap(0)

    def step(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x)
        self.graph.replay()
        return self.y


class DecodeStackGraph:
    """One decode step through a stack of layers as a single CUDA graph: the token
    rows go through ``layers[0].decode`` ... ``layers[-1].decode``, each layer's
    output feeding the next, with programmatic dependent launch across the whole
    stack, so a layer's projection weights start streaming while the previous
    layer finishes and no per-layer copy or graph launch sits between them.  The
    recurrent states and conv histories in ``states`` are updated in place."""

    def __init__(self, layers, states, B: int, overlap: bool = True):
        self.layers = list(layers)
        self.states = list(states)
        dev = self.states[0]["recurrent"].device
        self.x = torch.zeros(B, 1, self.layers[0].cfg.hidden, dtype=torch.bfloat16, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):                     # warm-up on scratch copies
            y = self.x
            for layer, st in zip(self.layers, self.states):
                scratch = {k_: v_.clone() for k_, v_ in st.items()}
                y, _ = layer.decode(y, scratch, scratch)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        lib = _lib.lib()
        lib.gdn_set_launch_overlap(1 if overlap else 0)
        try:
            with torch.cuda.graph(self.graph):
                y = self.x
                for layer, st in zip(self.layers, self.states):
                    y, _ = layer.decode(y, st, st)
                self.y = y
        finally:
            lib.gdn_set_launch_overlap(0)

    def step(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x)
        self.graph.replay()
        return self.y
