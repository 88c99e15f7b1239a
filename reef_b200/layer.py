"""Decoder layers over the C ABI: the Llama-shape W8A8 layer (BASELINE configs
3 and 4) and reef's GPT-Neo W8A8 block (configs 1 and 2), each on this rank's
tensor-parallel shard.

Weights are synthetic and seeded (there are no checkpoints here): fp32
N(0, 0.02) drawn on the device, quantised per output channel with reef's
quantize_rows (quant.hpp:112-133, run by the library's own quantiser, which
is bit-exact with it), then sharded by :mod:`reef_b200.tp`.  All compute
runs in libreef_b200.so; torch only holds device memory.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib, tp
from . import kernels as K


@dataclass(frozen=True)
class LlamaShape:
    hidden: int
    heads_q: int
    heads_kv: int
    ffn: int
    head_dim: int = 128
    rms_eps: float = 1e-5
    rope_base: float = 10000.0

    def ops_per_token(self, seq: int) -> dict:
        """Algorithmic int ops (2 per MAC) per token of a layer at full width;
        attention counts the causal (visible) half of q.k and p.v."""
        h, d = self.hidden, self.head_dim
        qkv = 2 * h * (self.heads_q + 2 * self.heads_kv) * d
        o = 2 * self.heads_q * d * h
        gu = 2 * h * 2 * self.ffn
        down = 2 * self.ffn * h
        attn = 2 * 2 * self.heads_q * d * (seq + 1) / 2
        return dict(gemm=qkv + o + gu + down, attention=attn)


# BASELINE.json configs 3 and 4
LLAMA_7B = LlamaShape(hidden=4096, heads_q=32, heads_kv=32, ffn=11008)
LLAMA_70B = LlamaShape(hidden=8192, heads_q=64, heads_kv=8, ffn=28672)


def _quantize_weight(w: torch.Tensor):
    """reef's per-output-channel quantize_rows on the device."""
    return K.quantize_rows(w.contiguous())


def _normal(gen, shape, std, device):
    return torch.randn(shape, generator=gen, device=device) * std


TP_ALLREDUCE = 0  # Megatron: replicated x / y, int32 partial sums all-reduced
TP_ALLGATHER = 1  # column-sharded x / y, int8 activations all-gathered


class LlamaLayer:
    """This rank's shard of one Llama-shape W8A8 decoder layer.

    tp_mode TP_ALLREDUCE: x / y are the full [tokens][hidden]; w_o and w_down
    hold this rank's input features (row-parallel).  TP_ALLGATHER: x / y are
    this rank's hidden/world columns; w_o and w_down hold this rank's output
    rows over the full K."""

    def __init__(self, shape: LlamaShape, batch: int, seq: int, seed: int = 0,
                 world: int = 1, rank: int = 0, comm: tp.Comm | None = None,
                 device: str | torch.device = "cuda", tp_mode: int = TP_ALLREDUCE):
        s = shape
        self.shape, self.batch, self.seq = s, batch, seq
        self.world, self.rank, self.comm = world, rank, comm
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        hq_l = s.heads_q // world
        hkv_l = s.heads_kv // world
        ffn_l = s.ffn // world
        if hq_l * world != s.heads_q or hkv_l * world != s.heads_kv or ffn_l * world != s.ffn:
            raise ValueError("heads and FFN must split evenly across the TP ranks")
        self.heads_q, self.heads_kv, self.ffn = hq_l, hkv_l, ffn_l
        d = s.head_dim
        std = 0.02

        def q_rows(full_rows, rows, k):
            w = _normal(g, (full_rows, k), std, dev)
            wq, ws = _quantize_weight(w)
            del w
            idx = torch.tensor(rows, device=dev)
            return wq.index_select(0, idx).contiguous(), ws.index_select(0, idx).contiguous()

        def q_cols(n, k_full, cols):
            w = _normal(g, (n, k_full), std, dev)
            wq, ws = _quantize_weight(w)  # full-row scales
            del w
            return wq[:, cols].contiguous(), ws

        self.attn_norm = torch.ones(s.hidden, device=dev)
        self.mlp_norm = torch.ones(s.hidden, device=dev)
        self.w_qkv, self.s_qkv = q_rows((s.heads_q + 2 * s.heads_kv) * d,
                                        tp.qkv_rows(s.heads_q, s.heads_kv, d, world, rank),
                                        s.hidden)
        self.tp_mode = tp_mode
        out_rows = list(range(*tp.shard_range(s.hidden, world, rank)))
        if tp_mode == TP_ALLGATHER:
            self.w_o, self.s_o = q_rows(s.hidden, out_rows, s.heads_q * d)
        else:
            self.w_o, self.s_o = q_cols(s.hidden, s.heads_q * d,
                                        tp.col_slice(s.heads_q * d, world, rank))
        self.w_gu, self.s_gu = q_rows(2 * s.ffn, tp.gate_up_rows(s.ffn, world, rank), s.hidden)
        if tp_mode == TP_ALLGATHER:
            self.w_down, self.s_down = q_rows(s.hidden, out_rows, s.ffn)
        else:
            self.w_down, self.s_down = q_cols(s.hidden, s.ffn, tp.col_slice(s.ffn, world, rank))
        torch.cuda.synchronize(dev)
        self.desc = _lib.LlamaLayerDesc(
            batch, seq, s.hidden, hq_l, hkv_l, d, ffn_l, s.rms_eps, s.rope_base,
            self.attn_norm.data_ptr(), self.w_qkv.data_ptr(), self.s_qkv.data_ptr(),
            self.w_o.data_ptr(), self.s_o.data_ptr(), self.mlp_norm.data_ptr(),
            self.w_gu.data_ptr(), self.s_gu.data_ptr(), self.w_down.data_ptr(),
            self.s_down.data_ptr(), comm.ptr if comm is not None else None, tp_mode)
        nbytes = _lib.lib().reef_b200_llama_layer_workspace_bytes(C.byref(self.desc))
        if nbytes == 0:
            raise ValueError("invalid Llama layer description")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    @property
    def tokens(self) -> int:
        return self.batch * self.seq

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None,
                stream: int | None = None) -> torch.Tensor:
        y = torch.empty_like(x) if out is None else out
        st = torch.cuda.current_stream().cuda_stream if stream is None else stream
        _lib.call("reef_b200_llama_layer_forward", C.byref(self.desc), x.data_ptr(),
                  y.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(), st)
        return y

    def alloc_cache(self, max_len: int) -> dict:
        """An empty int8 KV cache for `batch` sequences of this rank's KV heads:
        k / v [batch][heads_kv][max_len][128] int8 + per-(token, head) scales."""
        dev = self.w_qkv.device
        shp = (self.batch, self.heads_kv, max_len)
        return {"k": torch.zeros(shp + (128,), dtype=torch.int8, device=dev),
                "ks": torch.zeros(shp, device=dev),
                "v": torch.zeros(shp + (128,), dtype=torch.int8, device=dev),
                "vs": torch.zeros(shp, device=dev), "max_len": max_len}

    def _decode_tiles(self) -> None:
        """The four projections again in the decode layout
        (reef_b200_pack_weight_tiles), which the decode step's GEMMs stream
        as contiguous 16 KiB blocks; built on the first decode step."""
        lib = _lib.lib()
        self._tiles = {}
        for name, field in (("w_qkv", "t_qkv"), ("w_o", "t_o"), ("w_gu", "t_gu"),
                            ("w_down", "t_down")):
            w = getattr(self, name)
            rows, k = w.shape
            n = lib.reef_b200_weight_tiles_bytes(rows, k)
            buf = torch.empty(n + 1024, dtype=torch.uint8, device=w.device)
            off = (-buf.data_ptr()) % 1024
            ptr = buf.data_ptr() + off
            _lib.call("reef_b200_pack_weight_tiles", rows, k, w.data_ptr(), ptr,
                      torch.cuda.current_stream(w.device).cuda_stream)
            self._tiles[name] = buf
            setattr(self.desc, field, ptr)

    def decode(self, x: torch.Tensor, positions: torch.Tensor, cache: dict,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step: x [batch][hidden] (one new token per sequence) at
        `positions` (int32 [batch], device); appends to `cache`."""
        if getattr(self, "_tiles", None) is None:
            self._decode_tiles()
        max_len = cache["max_len"]
        ws = getattr(self, "_decode_ws", None)
        if ws is None or getattr(self, "_decode_len", None) != max_len:
            n = _lib.lib().reef_b200_llama_decode_workspace_bytes(C.byref(self.desc), max_len)
            if n == 0:
                raise ValueError("invalid decode description")
            self._decode_ws = ws = torch.empty(n, dtype=torch.uint8, device=x.device)
            self._decode_len = max_len
        y = torch.empty_like(x) if out is None else out
        _lib.call("reef_b200_llama_decode_forward", C.byref(self.desc), x.data_ptr(),
                  y.data_ptr(), positions.data_ptr(), cache["k"].data_ptr(),
                  cache["ks"].data_ptr(), cache["v"].data_ptr(), cache["vs"].data_ptr(), max_len,
                  ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        return y

    def host_weights(self) -> dict:
        """This rank's weights on the host (numpy), for the reference checks."""
        return {k: getattr(self, k).cpu().numpy() for k in
                ("attn_norm", "w_qkv", "s_qkv", "w_o", "s_o", "mlp_norm", "w_gu", "s_gu",
                 "w_down", "s_down")}


class GptNeoBlock:
    """This rank's shard of reef's GPT-Neo W8A8 block, from the block's float
    weights (numpy, the engine's [out][in] layout)."""

    def __init__(self, fw: dict, heads: int, seq: int, window: int = 0, eps: float = 1e-5,
                 world: int = 1, rank: int = 0, comm: tp.Comm | None = None,
                 device: str | torch.device = "cuda"):
        dev = torch.device(device)
        t = lambda a: torch.from_numpy(a).to(dev).contiguous()
        d = fw["wq"].shape[1]
        ffn = fw["wfc"].shape[0]
        hd = d // heads
        h0, h1 = tp.shard_range(heads, world, rank)
        f0, f1 = tp.shard_range(ffn, world, rank)
        rows = slice(h0 * hd, h1 * hd)

        def qrows(name, sl):
            wq, ws = _quantize_weight(t(fw[name]))
            return wq[sl].contiguous(), ws[sl].contiguous()

        def qcols(name, sl):
            wq, ws = _quantize_weight(t(fw[name]))
            return wq[:, sl].contiguous(), ws

        self.p = {}
        for n, s in (("wq", "sq"), ("wk", "sk"), ("wv", "sv")):
            self.p[n], self.p[s] = qrows(n, rows)
        self.p["wo"], self.p["so"] = qcols("wo", rows)
        self.p["wfc"], self.p["sfc"] = qrows("wfc", slice(f0, f1))
        self.p["wproj"], self.p["sproj"] = qcols("wproj", slice(f0, f1))
        for n in ("ln1_g", "ln1_b", "ln2_g", "ln2_b", "bo", "bproj"):
            self.p[n] = t(fw[n])
        self.p["bfc"] = t(fw["bfc"][f0:f1].copy())
        P = {k: v.data_ptr() for k, v in self.p.items()}
        self.desc = _lib.GptNeoBlockDesc(
            seq, d, h1 - h0, hd, f1 - f0, window, eps, P["ln1_g"], P["ln1_b"], P["wq"], P["sq"],
            P["wk"], P["sk"], P["wv"], P["sv"], P["wo"], P["so"], P["bo"], P["ln2_g"],
            P["ln2_b"], P["wfc"], P["sfc"], P["bfc"], P["wproj"], P["sproj"], P["bproj"],
            comm.ptr if comm is not None else None)
        nbytes = _lib.lib().reef_b200_gptneo_block_workspace_bytes(C.byref(self.desc))
        if nbytes == 0:
            raise ValueError("invalid GPT-Neo block description")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.seq, self.hidden = seq, d

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = torch.empty_like(x)
        _lib.call("reef_b200_gptneo_block_forward", C.byref(self.desc), x.data_ptr(),
                  y.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(),
                  torch.cuda.current_stream().cuda_stream)
        return y


class GptNeoModel:
    """A whole GPT-Neo (W8A8 or float) from reef's packed blob, generating on
    the GPU: the firmware's GptNeo (coral/firmware/gpt_neo.cc:61-188) over the
    C ABI.

    ``reef_b200_blob_load_model`` puts the blob's tables and layers in one
    device arena; ``step`` runs ``reef_b200_gptneo_step`` on ids already on
    the device, appending to the fp32 KV caches ([layers][max_tokens]
    [hidden] each); ``generate`` feeds each chosen id back on the device, so
    the loop reads nothing back until it ends.
    """

    def __init__(self, blob: bytes, max_tokens: int, device: str | torch.device = "cuda"):
        dev = torch.device(device)
        self._blob = C.create_string_buffer(bytes(blob), len(blob))
        self.info = _lib.BlobInfo()
        _lib.call("reef_b200_blob_read_info", self._blob, len(blob), C.byref(self.info))
        lib = _lib.lib()
        nbytes = lib.reef_b200_blob_model_bytes(C.byref(self.info))
        if nbytes == 0:
            raise ValueError("blob shape out of range")
        self.arena = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        w8a8 = self.info.precision == 1
        kind = _lib.GptNeoBlockDesc if w8a8 else _lib.GptNeoBlockF32Desc
        self.blocks = (kind * self.info.layers)()
        self.desc = _lib.GptNeoModelDesc()
        st = torch.cuda.current_stream(dev).cuda_stream
        _lib.call("reef_b200_blob_load_model", self._blob, len(blob), self.arena.data_ptr(),
                  nbytes, C.byref(self.desc), self.blocks if w8a8 else None,
                  None if w8a8 else self.blocks, st)
        if max_tokens > self.info.max_positions:
            raise ValueError("max_tokens past the position table")
        width = self.blocks[0].heads * self.blocks[0].head_dim
        shape = (self.info.layers, max_tokens, width)
        self.k_cache = torch.zeros(shape, dtype=torch.float32, device=dev)
        self.v_cache = torch.zeros(shape, dtype=torch.float32, device=dev)
        self.max_tokens = max_tokens
        wbytes = lib.reef_b200_gptneo_step_workspace_bytes(C.byref(self.desc), max_tokens)
        if wbytes == 0:
            raise ValueError("invalid model description")
        self.workspace = torch.empty(wbytes, dtype=torch.uint8, device=dev)
        self.position = 0
        self.device = self.arena.device  # with its index

    def step(self, ids: torch.Tensor, logits: torch.Tensor | None = None,
             next_id: torch.Tensor | None = None) -> None:
        """Runs ``ids`` (device uint32/int32 [count]) at the next positions;
        writes the last one's logits and greedy id where given."""
        if ids.dtype not in (torch.int32, torch.uint32) or not ids.is_contiguous() or \
                ids.device != self.device:
            raise TypeError("ids must be a contiguous 32-bit integer tensor on the model's device")
        count = ids.numel()
        _lib.call("reef_b200_gptneo_step", C.byref(self.desc), ids.data_ptr(), count,
                  self.position, self.k_cache.data_ptr(), self.v_cache.data_ptr(),
                  self.max_tokens, logits.data_ptr() if logits is not None else None,
                  next_id.data_ptr() if next_id is not None else None,
                  self.workspace.data_ptr(), self.workspace.numel(),
                  torch.cuda.current_stream(self.device).cuda_stream)
        self.position += count

    def generate(self, prompt, new_tokens: int):
        """Greedy generation (GPTNeo::generate): the prompt at once, then one
        token a time.  Returns (tokens [new_tokens] int64, logits
        [new_tokens][vocab]), the logits behind each token."""
        dev = self.device
        ids = torch.tensor(list(prompt), dtype=torch.int32, device=dev)
        tokens = torch.empty(new_tokens, dtype=torch.int32, device=dev)
        logits = torch.empty((new_tokens, self.info.vocab), dtype=torch.float32, device=dev)
        self.step(ids, logits[0], tokens[0:1])
        for i in range(1, new_tokens):
            self.step(tokens[i - 1:i], logits[i], tokens[i:i + 1])
        return tokens.to(torch.int64).cpu(), logits.cpu()
