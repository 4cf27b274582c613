"""Dual-AR decode frame driver on the device.

One frame is the reference's ``DecodeGraphs.decode`` + ``sample_frame``
(app/engine/graphs.py:92-132, :205-217, :348-355), replayed as ONE captured
CUDA graph with no host round trip:

  slow AR: 36 decode blocks at the device-side position  (fusedlayer.decode_block)
  final RMSNorm, bf16 LM head over the vocabulary         (heads.dense_linear)
  main token: top-k / top-p sample; repetition-aware resample with a hotter
  setting when the main token repeats within the window   (heads.sample)
  fast AR prime at fast position 0 with the slow hidden state: every fast
  block but the last, and the last block's q/k/v projection + rotary + KV
  write only (its attention output feeds nothing: app/engine/graphs.py:76-89)
  9 fast steps: codebook embedding -> 4 fast blocks -> norm -> codebook head
  -> sample
  next frame's input: semantic embedding + the frame's codebook embeddings;
  position and draw counters advance on the device.

The model is random-init NF4 with S2-Pro dimensions (the checkpoint is not
available): weights N(0, 0.02), norm weights N(1, 0.1), embeddings N(0, 1)
scaled by 0.02 - or loaded from a state dict (``state_dict()`` /
``DualARDecoder(..., state_dict=sd)``), whose NF4 blocks use bitsandbytes'
serialisation (ttspipe_b200.checkpoint). The prompt is prefilled through the same blocks (GEMM path,
the grouped attention of app/engine/fastpath.py:158-174).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from ttspipe_b200 import _lib, checkpoint, fusedlayer, fusedops, heads, nf4gemv
from ttspipe_b200.model import ModelArgs, precompute_freqs_cis, random_block


@dataclass
class DualARConfig:
    slow: ModelArgs = field(default_factory=lambda: ModelArgs(n_layer=36, max_seq_len=2048))
    n_fast_layer: int = 4
    vocab: int = 155136
    num_codebooks: int = 10
    codebook_size: int = 4096
    semantic_begin_id: int = 151040        # the codebook-0 tokens: [begin, begin + codebook_size)
    temperature: float = 0.7
    top_p: float = 0.8
    top_k: int = 64
    high_temperature: float = 1.0          # repetition-aware resample (app/engine/graphs.py:105-116)
    high_top_p: float = 0.9
    ras_window: int = 16


class DualARDecoder:
    """A Dual-AR model on one GPU (random-init, or from a state dict) and its
    captured frame graph. `seed` also seeds the draws."""

    def __init__(self, cfg: DualARConfig, device, seed: int = 0, n_slow: int | None = None,
                 state_dict: dict | None = None):
        if not (nf4gemv.available() and nf4gemv.install() and fusedlayer.install() and fusedops.install()):
            raise RuntimeError("the sm_100a kernels are not available")
        self.cfg, self.device, self.seed = cfg, torch.device(device), seed
        sc = cfg.slow
        n_slow = sc.n_layer if n_slow is None else n_slow
        g = torch.Generator(device=self.device).manual_seed(seed)

        def randn(*shape, std=0.02):
            return (torch.randn(*shape, generator=g, device=self.device) * std).to(torch.bfloat16)

        def norm_w():
            return (1.0 + 0.1 * torch.randn(sc.dim, generator=g, device=self.device)).to(torch.bfloat16)

        fast_args = ModelArgs(dim=sc.dim, n_head=sc.n_head, n_local_heads=sc.n_local_heads, head_dim=sc.head_dim,
                              intermediate_size=sc.intermediate_size, max_seq_len=16, n_layer=cfg.n_fast_layer,
                              attention_qk_norm=sc.attention_qk_norm, norm_eps=sc.norm_eps, rope_base=sc.rope_base)
        self.fast_args = fast_args
        if state_dict is None:
            self.slow = [random_block(sc, device=self.device, seed=seed * 1000 + i) for i in range(n_slow)]
            self.fast = [random_block(fast_args, device=self.device, seed=seed * 1000 + 500 + i)
                         for i in range(cfg.n_fast_layer)]
        else:
            self.slow = [checkpoint.load_block(state_dict, f"layers.{i}", sc, self.device) for i in range(n_slow)]
            self.fast = [checkpoint.load_block(state_dict, f"fast_layers.{i}", fast_args, self.device)
                         for i in range(cfg.n_fast_layer)]
        for blk in self.slow + self.fast:
            for lin in (blk.attention.wqkv, blk.attention.wo, blk.feed_forward.w1, blk.feed_forward.w3,
                        blk.feed_forward.w2):
                assert nf4gemv.prepare(lin)
        self.norm_w, self.fast_norm_w = norm_w(), norm_w()
        self.lm_head = randn(cfg.vocab, sc.dim)
        self.cb_heads = [randn(cfg.codebook_size, sc.dim) for _ in range(cfg.num_codebooks)]
        self.sem_emb = randn(cfg.vocab, sc.dim)
        self.cb_emb = randn(cfg.num_codebooks, cfg.codebook_size, sc.dim)
        self.fast_emb = randn(cfg.codebook_size, sc.dim)
        if state_dict is not None:
            self._load_dense(state_dict)
        self.freqs = precompute_freqs_cis(sc.max_seq_len, sc.head_dim, sc.rope_base, device=self.device)
        self.fast_freqs = precompute_freqs_cis(16, sc.head_dim, sc.rope_base, device=self.device)
        self.mask = torch.ones(1, 1, 1, sc.max_seq_len, dtype=torch.bool, device=self.device)
        self.fast_mask = torch.ones(1, 1, 1, 16, dtype=torch.bool, device=self.device)
        # device state of the frame loop
        self.pos = torch.zeros(1, dtype=torch.long, device=self.device)
        self.step = torch.zeros(1, dtype=torch.long, device=self.device)
        self.fast_pos = [torch.full((1,), i, dtype=torch.long, device=self.device)
                         for i in range(cfg.num_codebooks)]
        self.draw = [torch.zeros(1, dtype=torch.long, device=self.device) for _ in range(cfg.num_codebooks + 1)]
        self.x = torch.zeros(1, 1, sc.dim, dtype=torch.bfloat16, device=self.device)
        self.tokens = torch.zeros(cfg.num_codebooks + 1, dtype=torch.long, device=self.device)
        self.recent = torch.full((cfg.ras_window,), -1, dtype=torch.long, device=self.device)
        self.main_tok = torch.zeros(1, dtype=torch.long, device=self.device)   # the two semantic draws
        self.high_tok = torch.zeros(1, dtype=torch.long, device=self.device)
        self.h = torch.zeros(1, 1, sc.dim, dtype=torch.bfloat16, device=self.device)  # the fast AR's input
        # the frame's logit rows (the LM head's and each codebook head's), kept
        # in place so a replayed graph writes the same buffers every frame
        self.logits = torch.zeros(cfg.vocab, dtype=torch.bfloat16, device=self.device)
        self.cb_logits = torch.zeros(cfg.num_codebooks, cfg.codebook_size, dtype=torch.bfloat16, device=self.device)
        self.graph = None

    # ------------------------------------------------------------------ checkpoint
    # Names: the fork's module lists model.layers / model.fast_layers
    # (app/engine/graphs.py:86-88, app/engine/cpu.py:236-252) and its tables
    # model.embeddings and model.codebook_embeddings, flat
    # [num_codebooks * codebook_size, dim] (app/engine/hostembed.py:3-4,
    # app/engine/streamgen.py:269); the rest are this decoder's: fast_embeddings,
    # norm, fast_norm, output (the LM head) and fast_output.{i} (codebook i's head).
    def state_dict(self) -> dict:
        """The model as a checkpoint state dict (NF4 blocks in bitsandbytes'
        serialisation, dense tensors as they are)."""
        cfg = self.cfg
        sd = {}
        for i, blk in enumerate(self.slow):
            sd.update(checkpoint.block_state_dict(blk, f"layers.{i}"))
        for i, blk in enumerate(self.fast):
            sd.update(checkpoint.block_state_dict(blk, f"fast_layers.{i}"))
        sd["embeddings.weight"] = self.sem_emb
        sd["codebook_embeddings.weight"] = self.cb_emb.reshape(cfg.num_codebooks * cfg.codebook_size, -1)
        sd["fast_embeddings.weight"] = self.fast_emb
        sd["norm.weight"] = self.norm_w
        sd["fast_norm.weight"] = self.fast_norm_w
        sd["output.weight"] = self.lm_head
        for i, h in enumerate(self.cb_heads):
            sd[f"fast_output.{i}.weight"] = h
        return sd

    @torch.no_grad()
    def _load_dense(self, sd) -> None:
        cfg, dim = self.cfg, self.cfg.slow.dim

        def take(name, shape):
            t = sd.get(name)
            if t is None:
                raise ValueError(f"missing {name}")
            if tuple(t.shape) != tuple(shape):
                raise ValueError(f"{name} is {tuple(t.shape)}, expected {tuple(shape)}")
            return t.to(self.device, torch.bfloat16).contiguous()

        self.sem_emb = take("embeddings.weight", (cfg.vocab, dim))
        self.cb_emb = take("codebook_embeddings.weight", (cfg.num_codebooks * cfg.codebook_size, dim)).view(
            cfg.num_codebooks, cfg.codebook_size, dim)
        self.fast_emb = take("fast_embeddings.weight", (cfg.codebook_size, dim))
        self.norm_w = take("norm.weight", (dim,))
        self.fast_norm_w = take("fast_norm.weight", (dim,))
        self.lm_head = take("output.weight", (cfg.vocab, dim))
        self.cb_heads = [take(f"fast_output.{i}.weight", (cfg.codebook_size, dim)) for i in range(cfg.num_codebooks)]

    # ------------------------------------------------------------------ prompt
    @torch.no_grad()
    def prefill(self, prompt_ids: torch.Tensor) -> None:
        """Run the prompt through the slow stack (filling its KV caches) and set
        the first frame's input to the last prompt position's embedding."""
        n = prompt_ids.numel()
        sc = self.cfg.slow
        x = self.sem_emb.index_select(0, prompt_ids.to(self.device)).view(1, n, sc.dim)
        pos = torch.arange(n, device=self.device)
        mask = torch.tril(torch.ones(n, sc.max_seq_len, dtype=torch.bool, device=self.device)).view(1, 1, n, -1)
        freqs = self.freqs[:n]
        for blk in self.slow:
            x = blk(x, freqs, mask, pos)
        self.x.copy_(self.sem_emb[prompt_ids[-1]].view(1, 1, -1))
        self.pos.fill_(n)
        self.step.zero_()

    # ------------------------------------------------------------------ frame
    def _fast_prime(self, hidden) -> None:
        """Fast position 0 for its KV entries only: the last block's attention
        output and feed-forward feed nothing, so only its q/k/v projection,
        rotary and KV write run."""
        x = hidden
        for blk in self.fast[:-1]:
            x = fusedlayer.decode_block(blk, x, self.fast_freqs[0:1], self.fast_mask, self.fast_pos[0])
        last = self.fast[-1]
        a = last.attention
        xn = fusedops.rms_norm(x, last.attention_norm.weight, last.attention_norm.eps)
        qkv = nf4gemv.matmul(a.wqkv, xn)
        q = torch.empty(a.n_head * a.head_dim, dtype=torch.bfloat16, device=self.device)
        st = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(_lib.lib().nf4b_qk_rope_kv(
            qkv.data_ptr(), None, None, 1e-6, self.fast_freqs.data_ptr(), _lib.NF4B_BF16, self.fast_pos[0].data_ptr(),
            q.data_ptr(), a.kv_cache.k_cache.data_ptr(), a.kv_cache.v_cache.data_ptr(), a.n_head, a.n_local_heads,
            a.head_dim, a.kv_cache.k_cache.shape[2], st))

    @torch.no_grad()
    def slow_stack(self, x):
        """The slow blocks at the device-side position `self.pos` (capturable):
        the rotary row is gathered on the device, so a replayed graph rotates
        q and k for the position of the frame it runs, the way the
        reference's model indexes ``freqs_cis[input_pos]`` before its layers."""
        fr = self.freqs.index_select(0, self.pos)
        for i, blk in enumerate(self.slow):
            nxt = self.slow[i + 1] if i + 1 < len(self.slow) else None
            x = fusedlayer.decode_block(blk, x, fr, self.mask, self.pos, next_block=nxt)
            assert x is not None, "a slow block fell back"
        return x

    @torch.no_grad()
    def frame(self) -> None:
        """Issue one frame on the current stream (capturable)."""
        cfg = self.cfg
        x = self.slow_stack(self.x)
        hidden = fusedops.rms_norm(x, self.norm_w, cfg.slow.norm_eps)
        logits = heads.dense_linear(self.lm_head, hidden, out=self.logits)
        heads.sample(logits, temperature=cfg.temperature, top_p=cfg.top_p, top_k=cfg.top_k,
                     seed=self.seed * 7919 + 1, step=self.step, out=self.main_tok)
        heads.sample(logits, temperature=cfg.high_temperature, top_p=cfg.high_top_p, top_k=cfg.top_k,
                     seed=self.seed * 7919 + 2, step=self.step, out=self.high_tok)
        L = _lib.lib()
        st = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        dim = self.h.shape[-1]
        # the repetition-aware choice (app/engine/graphs.py:111-116), tokens[0..1]
        # and the fast AR's first input, in one launch
        _lib.check(L.nf4b_frame_select(self.main_tok.data_ptr(), self.high_tok.data_ptr(), self.recent.data_ptr(),
                                       self.recent.numel(), cfg.semantic_begin_id, cfg.codebook_size,
                                       self.tokens.data_ptr(), self.fast_emb.data_ptr(), dim, self.h.data_ptr(), st))
        self._fast_prime(hidden)
        for i in range(1, cfg.num_codebooks):
            y = self.h
            for blk in self.fast:
                y = fusedlayer.decode_block(blk, y, self.fast_freqs[i:i + 1], self.fast_mask, self.fast_pos[i])
                assert y is not None, "a fast block fell back"
            # fast_norm folded into the codebook head's launch
            logits_i = heads.dense_linear(self.cb_heads[i], y, out=self.cb_logits[i],
                                          norm=(self.fast_norm_w, cfg.slow.norm_eps))
            tok = self.tokens[i + 1:i + 2]
            heads.sample(logits_i, temperature=cfg.temperature, top_p=cfg.top_p, top_k=cfg.top_k,
                         seed=self.seed * 7919 + 10 + i, step=self.step, out=tok)
            _lib.check(L.nf4b_embed_rows(self.fast_emb.data_ptr(), self.fast_emb.shape[0], tok.data_ptr(), 1, dim,
                                         self.h.data_ptr(), st))
        # next frame's input (semantic + codebook embeddings) and counters, one launch
        _lib.check(L.nf4b_frame_advance(self.sem_emb.data_ptr(), self.sem_emb.shape[0], self.cb_emb.data_ptr(),
                                        cfg.codebook_size, cfg.num_codebooks, self.tokens.data_ptr(), dim,
                                        self.x.data_ptr(), self.recent.data_ptr(), self.recent.numel(),
                                        self.pos.data_ptr(), self.step.data_ptr(), st))

    def capture(self) -> None:
        """Record one frame as a CUDA graph (state lives in device tensors)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        saved = (self.pos.clone(), self.step.clone(), self.x.clone(), self.recent.clone())
        with torch.cuda.stream(s):
            self.frame()              # eager pass: sizes every workspace before capture
            torch.cuda.synchronize(self.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self.frame()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.pos.copy_(saved[0])
        self.step.copy_(saved[1])
        self.x.copy_(saved[2])
        self.recent.copy_(saved[3])

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        self.graph = None
