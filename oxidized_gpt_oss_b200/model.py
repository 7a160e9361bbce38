"""Full decoder — mirror of GPTModel (src/model.rs) and the greedy loop of
InferenceEngine (src/inference.rs) of the reference.

* ``GPTModel.forward(input_ids)`` replaces ``GPTModel::forward(&self,
  input_ids: &[u32], _position_ids) -> Result<MetalBuffer>``
  (src/model.rs:713-741): the tokens are appended to the KV cache and the
  last token's logits are returned (f32 here; the reference returns f16).
* ``GPTModel.reset_kv_cache()`` replaces src/model.rs:743-747.
* ``GPTModel.generate(prompt, max_tokens)`` is ``generate_chat``'s loop at
  temperature 0 (src/inference.rs:62-97) without the tokenizer: reset, one
  prefill of the prompt, then one token per step, each the argmax of the
  previous logits (ties to the last index, src/sampler.rs:7-16), fed back on
  the device.

Every layer runs in liboxg_b200.so: attention (oxg_model_*) and the MoE block
(oxg_moe_upload per layer). There is no host fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import abi

_ATTN_KEYS = ("attn_norm", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "bo", "sinks", "mlp_norm")


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        return a.data_ptr()
    return a.ctypes.data


def _contig(a):
    if isinstance(a, np.ndarray):
        return np.ascontiguousarray(a)
    if isinstance(a, torch.Tensor):
        return a.contiguous()
    return a


class GPTModel:
    """A gpt-oss-architecture decoder resident on one GPU.

    ``weights`` is the dict of ``synth.model_weights`` (numpy or torch, host or
    CUDA): ``dims``, ``embed``, ``unembed``, ``final_norm`` and ``layers`` (per
    layer the attention arrays of ``_ATTN_KEYS`` and ``moe``, an MoE-block dict).
    """

    def __init__(self, weights: dict, *, max_seq: int = 4096, max_tokens: int = 2048, max_batch: int = 1,
                 ctx: abi.Context | None = None, experts: tuple[int, int] | None = None, kv_pages: int = 0):
        """experts: (begin, count) to keep only that range of every MoE
        block's experts (expert parallelism; then ``connect_expert_parallel``
        on every process before the first forward). kv_pages: pages of 64
        positions in the KV-cache pool the sequences share (0: room for every
        sequence at max_seq)."""
        # a context of its own (its layer ids 0..n_layers-1 must not collide
        # with other MoE layers), bound to torch's current stream
        self.ctx = ctx if ctx is not None else abi.Context(torch.cuda.current_device())
        self.ctx.set_stream(torch.cuda.current_stream())
        d = weights["dims"]
        self.dims = dict(d)
        self.vocab = int(d["vocab"])
        self.n_layers = int(d["n_layers"])
        self.max_seq = int(max_seq)
        self.max_tokens = int(min(max_tokens, max_seq))
        md = abi.ModelDims(self.n_layers, int(d["hidden"]), int(d["n_heads"]), int(d["n_kv_heads"]),
                           int(d["head_dim"]), self.vocab, int(d["sliding_window"]), self.max_seq,
                           self.max_tokens, float(d["rope_theta"]), float(d["rms_eps"]), int(max_batch),
                           int(kv_pages))
        self.max_batch = max(int(max_batch), 1)
        lib, h = self.ctx.lib, self.ctx.handle
        abi.check(lib.oxg_model_init(h, ctypes.byref(md)), h)
        e, u, n = (_contig(weights[k]) for k in ("embed", "unembed", "final_norm"))
        abi.check(lib.oxg_model_upload_embeddings(h, _ptr(e), _ptr(u), _ptr(n)), h)
        for layer, lw in enumerate(weights["layers"]):
            keep = {k: _contig(lw.get(k)) for k in _ATTN_KEYS}
            aw = abi.AttnWeights(*[_ptr(keep[k]) for k in _ATTN_KEYS])
            abi.check(lib.oxg_model_upload_attention(h, layer, ctypes.byref(aw)), h)
            mw = lw["moe"]
            mkeep = {k: _contig(mw.get(k)) for k in ("router_w", "router_b", "w1_blocks", "w1_scales", "b1",
                                                     "w2_blocks", "w2_scales", "b2")}
            dims = abi.MoeDims(int(mw["hidden"]), int(mw["intermediate"]), int(mw["n_experts"]),
                               int(mw["top_k"]), float(mw["alpha"]), float(mw["limit"]))
            ws = abi.MoeWeights(*[_ptr(mkeep[k]) for k in ("router_w", "router_b", "w1_blocks", "w1_scales",
                                                            "b1", "w2_blocks", "w2_scales", "b2")])
            if experts is None:
                abi.check(lib.oxg_moe_upload(h, layer, ctypes.byref(dims), ctypes.byref(ws)), h)
            else:
                abi.check(lib.oxg_moe_upload_shard(h, layer, ctypes.byref(dims), ctypes.byref(ws),
                                                   int(experts[0]), int(experts[1])), h)
        self.experts = experts
        self._ep = None
        self._moe_hidden = int(weights["layers"][0]["moe"]["hidden"])
        dev = torch.device("cuda", self.ctx.device)
        self._dev = dev
        self._topk = int(weights["layers"][0]["moe"]["top_k"])
        self._tap = None

    def connect_expert_parallel(self, group=None, max_recv_rows: int = 0) -> None:
        """Expert parallelism over NVLink peer memory for every MoE block (all
        layers share one exchange: the buffers depend only on the shapes and
        the expert range). Collective over ``group``: every process, with the
        shard ``ep.shard_range`` gives its rank, calls it once; afterwards
        every process must run the same forwards / batched steps (the MoE
        blocks exchange rows with the others), eagerly: ``decode`` and
        ``generate`` capture CUDA graphs and refuse shard layers."""
        from types import SimpleNamespace
        from .ep import PeerExpertParallelMoE
        if self.experts is None:
            raise ValueError("the model holds whole MoE blocks: construct it with experts=(begin, count)")
        shard = SimpleNamespace(ctx=self.ctx, layer=0, hidden=self._moe_hidden)
        # batched decode steps (one token per sequence) receive on the grouped
        # decode kernels; prompt chunks on the prefill GEMMs
        self._ep = PeerExpertParallelMoE(shard, max_tokens=self.max_tokens, group=group,
                                         max_recv_rows=max_recv_rows, decode_tokens=min(self.max_batch, 64))

    def close_expert_parallel(self) -> None:
        if self._ep is not None:
            self._ep.close()
            self._ep = None

    # -- reference-shaped API ------------------------------------------------
    def reset_kv_cache(self) -> None:
        abi.check(self.ctx.lib.oxg_model_reset(self.ctx.handle), self.ctx.handle)

    def reset_sequence(self, seq: int) -> None:
        """Empties sequence ``seq``'s cache and returns its pages to the pool."""
        abi.check(self.ctx.lib.oxg_model_reset_seq(self.ctx.handle, int(seq)), self.ctx.handle)

    def kv_pages(self) -> tuple[int, int]:
        """(pages in use, pages in the pool) of the paged KV cache."""
        used, total = ctypes.c_int(), ctypes.c_int()
        abi.check(self.ctx.lib.oxg_model_kv_pages(self.ctx.handle, ctypes.byref(used), ctypes.byref(total)),
                  self.ctx.handle)
        return used.value, total.value

    def position(self) -> int:
        p = ctypes.c_int()
        abi.check(self.ctx.lib.oxg_model_position(self.ctx.handle, ctypes.byref(p)), self.ctx.handle)
        return p.value

    def forward(self, input_ids, n_logits: int = 1) -> torch.Tensor:
        """Appends ``input_ids`` to the cache; returns f32 logits [n_logits, V]
        of the last n_logits tokens (one row, like the reference, by default)."""
        ids = torch.as_tensor(np.asarray(input_ids, dtype=np.int32)).to(self._dev)
        if ids.numel() > 0 and (int(ids.min()) < 0 or int(ids.max()) >= self.vocab):
            bad = int(ids.max()) if int(ids.max()) >= self.vocab else int(ids.min())
            raise abi.OxgError(abi.OXG_ERR_INVALID_ARG, f"Token id {bad} out of bounds")
        logits = torch.empty((n_logits, self.vocab), dtype=torch.float32, device=self._dev)
        nxt = torch.empty((max(n_logits, 1),), dtype=torch.int32, device=self._dev)
        self.forward_device(ids, n_logits, logits, nxt)
        return logits

    def forward_device(self, ids: torch.Tensor, n_logits: int, logits: torch.Tensor | None,
                       nxt: torch.Tensor | None) -> None:
        """Device-side forward (no host synchronisation): ids int32 CUDA tensor."""
        abi.check(self.ctx.lib.oxg_model_forward(self.ctx.handle, ids.data_ptr(), int(ids.numel()), int(n_logits),
                                                 _ptr(logits), _ptr(nxt)), self.ctx.handle)

    def prefill_seq(self, seq: int, input_ids) -> torch.Tensor:
        """Appends a prompt (at most max_tokens ids) to sequence ``seq``'s own
        KV cache; returns its greedy next token (int32 CUDA tensor [1])."""
        if isinstance(input_ids, torch.Tensor):
            ids = input_ids.to(device=self._dev, dtype=torch.int32).contiguous()
        else:
            ids = torch.as_tensor(np.asarray(input_ids, dtype=np.int32)).to(self._dev)
        nxt = torch.empty(1, dtype=torch.int32, device=self._dev)
        abi.check(self.ctx.lib.oxg_model_prefill_seq(self.ctx.handle, int(seq), ids.data_ptr(), int(ids.numel()),
                                                     nxt.data_ptr()), self.ctx.handle)
        return nxt

    def step_batch(self, tokens: torch.Tensor, logits: torch.Tensor | None = None) -> torch.Tensor:
        """One token for each of sequences 0 .. len(tokens)-1 as one batch
        (each attends to its own cache); returns their greedy next tokens
        (int32 CUDA tensor) and fills ``logits`` [len(tokens), V] f32 if given."""
        tok = tokens.to(device=self._dev, dtype=torch.int32).contiguous()
        nxt = torch.empty(tok.numel(), dtype=torch.int32, device=self._dev)
        abi.check(self.ctx.lib.oxg_model_step_batch(self.ctx.handle, int(tok.numel()), tok.data_ptr(),
                                                    nxt.data_ptr(), _ptr(logits)), self.ctx.handle)
        return nxt

    def decode(self, n_steps: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """n_steps greedy one-token steps on the device (a captured CUDA graph
        replayed per token), continuing from the last forward's greedy token;
        returns the new tokens (int32 CUDA tensor) without synchronising."""
        if out is None:
            out = torch.empty((max(int(n_steps), 1),), dtype=torch.int32, device=self._dev)
        abi.check(self.ctx.lib.oxg_model_decode(self.ctx.handle, int(n_steps), out.data_ptr()), self.ctx.handle)
        return out[:n_steps]

    def route_tap(self, max_tokens: int | None) -> torch.Tensor | None:
        """Starts recording each layer's chosen experts for forwards of up to
        max_tokens tokens (None stops): returns the int32 CUDA buffer
        [n_layers, max_tokens, k] that every forward overwrites."""
        if max_tokens is None:
            abi.check(self.ctx.lib.oxg_model_route_tap(self.ctx.handle, None, 0), self.ctx.handle)
            self._tap = None
            return None
        k = int(self._topk)
        self._tap = torch.full((self.n_layers, int(max_tokens), k), -1, dtype=torch.int32, device=self._dev)
        abi.check(self.ctx.lib.oxg_model_route_tap(self.ctx.handle, self._tap.data_ptr(), int(max_tokens)),
                  self.ctx.handle)
        return self._tap

    def generate(self, prompt, max_tokens: int) -> list[int]:
        """Greedy generation through ``oxg_model_generate`` (host arrays)."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        out = np.empty(int(max_tokens), dtype=np.int32)
        abi.check(self.ctx.lib.oxg_model_generate(self.ctx.handle, p.ctypes.data, int(p.size), int(max_tokens),
                                                  out.ctypes.data), self.ctx.handle)
        return out.tolist()

    def sync(self) -> None:
        self.ctx.sync()

    def release(self) -> None:
        if self.ctx is not None and self.ctx.handle:
            self.ctx.lib.oxg_model_release(self.ctx.handle)
            for layer in range(self.n_layers):
                self.ctx.lib.oxg_moe_release(self.ctx.handle, layer)
