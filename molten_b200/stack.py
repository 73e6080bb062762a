"""The stacked decode loop of BASELINE cfg4 on the decode kernels.

One decode step for a batch of B tokens (rows x [B, 2048], each the
embedding row of the token being decoded):

    for each of the L layers:
        p   = proj_l(x)                             Q4 2048x2048 GEMV (gemv_quant)
        out = MoE_l(h = x, b = p)                   add + RMSNorm + router + top-4 +
                                                    SwiGLU experts + weighted combine
        x   = out
    key   = argmax over the Q6 LM head of x         gemv_head_argmax
    token = key's index; x = embed[token]           token_tail (reads and clears key)

The MoE layer normalises its input (RMSNorm of h + b) before the router and
the experts, so activations stay bounded over the stack without a separate
residual stream. The expert part runs one of three ways (``moe_path``):

  "fused"    B = 1: the one-launch fused layer, the default at batch 1;
             with ``fuse_proj`` (the default) the layer's projection runs
             inside the same launch (moe_decode_layer_proj: one launch per
             layer, bit-identical to gemv_quant + moe_decode_layer);
  "grouped"  B > 1: router_addnorm_route for the B rows, then the prefill
             MoE FFN (moe_prefill: route, sort, gather, tensor-core grouped
             GEMMs, combine), so each routed expert's rows are read and
             dequantised once per step for all of its tokens -- the default
             above B = 16 (measured on B200: 2439 vs 1987 tokens/s for "gemv"
             vs "grouped" at B = 16, 2473 vs 3123 at B = 32); activations match the oracle within the prefill
             tolerance, the ids given the same logits bit for bit;
  "gemv"     any B: router_addnorm_route, gemv_gather_act and
             gemv_gather_down_combine4, per-token GEMVs bit-identical to the
             oracle -- the default for 1 < B <= 16.

The token feeds back on the device, so a step can be captured once in a CUDA
graph and replayed.

With ``sampling`` (batch 1, the reference's temperature > 0 path,
lfm/sample.rs), the head stores its bf16 logits (gemv_quant) and the draw
(mc_sample_draw) folds the sampled token into the same key the greedy head
writes; the token tail then runs unchanged and mc_sample_mark adds the token
to the seen set and advances the device position, so the sampled step is
graph-capturable too.
"""
from __future__ import annotations

import torch

from molten_b200 import lfm


class DecodeStack:
    def __init__(self, ctx: lfm.Context, layers: list[dict], head, embed: torch.Tensor,
                 batch: int, n_experts: int = 64, moe_path: str | None = None, sampling=None,
                 fuse_proj: bool = True):
        self.ctx, self.layers, self.head, self.embed = ctx, layers, head, embed
        self.sampling = sampling
        lfm.ensure(sampling is None or batch == 1, "sampling decodes one sequence")
        self.B, self.E = batch, n_experts
        # measured on B200 (40 layers): batch 8 runs faster on the per-token
        # GEMVs, batch 32 on the grouped expert GEMMs
        self.path = moe_path or ("fused" if batch == 1 else "gemv" if batch <= 16 else "grouped")
        lfm.ensure(self.path in ("fused", "grouped", "gemv"), f"moe_path {self.path!r}")
        lfm.ensure(self.path != "fused" or batch == 1, "the fused layer is batch 1")
        self.fuse_proj = fuse_proj and self.path == "fused"
        H = embed.shape[1]
        I = layers[0]["gate"].out_features // n_experts
        dev = embed.device
        bf = lambda *s: torch.empty(s, dtype=torch.bfloat16, device=dev)
        i32 = lambda *s: torch.zeros(s, dtype=torch.int32, device=dev)
        self.x = bf(batch, H)                    # step input: embedding rows
        self.p, self.hout, self.normed = bf(batch, H), bf(batch, H), bf(batch, H)
        self.outs = (bf(batch, H), bf(batch, H))
        self.logits = torch.empty((batch, n_experts), dtype=torch.float32, device=dev)
        self.ids = [i32(batch, 4) for _ in layers]
        self.wts = [bf(batch, 4) for _ in layers]
        self.counter = i32(batch)
        self.act = bf(batch, 4, I)
        self.keys = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.tokens = i32(batch)
        self.tail_norm_w = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.tail_normed = bf(batch, H)
        self.ws = None
        if self.path == "fused":
            words = (lfm.moe_decode_proj_workspace_words(I) if self.fuse_proj
                     else lfm.moe_decode_workspace_words(I))
            self.ws = torch.zeros(words, dtype=torch.int32, device=dev)
        self.pws = None
        if self.path == "grouped":
            nb = lfm.moe_prefill_workspace_size(batch, n_experts, H, I)
            self.pws = torch.zeros(nb, dtype=torch.uint8, device=dev)
        self.sample = None
        if sampling is not None:
            from molten_b200.sample import SampleScratch
            self.sample = SampleScratch(ctx, head.out_features)
            self.head_logits = bf(head.out_features)
            self.pos = torch.zeros(1, dtype=torch.int32, device=dev)

    def start(self, tokens: torch.Tensor, pos: int = 0, seen=()) -> None:
        """Loads the embedding rows of the first tokens (int32 [B]); with
        sampling, ``pos`` is the absolute position of the token the next step
        draws and ``seen`` the sequence's token ids so far."""
        self.x.copy_(self.embed[tokens.long()])
        if self.sample is not None:
            self.pos.fill_(pos)
            self.sample.upload_seen(list(seen) + [int(t) for t in tokens.cpu()])

    def step(self) -> None:
        ctx, cur = self.ctx, self.x
        for l, L in enumerate(self.layers):
            nxt = self.outs[l % 2]
            if self.fuse_proj:
                # the next layer's router rows and projection codes into L2
                # while this layer exchanges its act rows (its norm weights
                # are read before the launch's dependency wait anyway)
                following = self.layers[(l + 1) % len(self.layers)]
                ctx.prefetch_next(following["router"], following["proj"].codes)
                lfm.moe_decode_layer_proj(ctx, cur, L["proj"], L["norm_w"], self.hout, self.normed,
                                          L["router"], self.logits, None, self.ids[l],
                                          self.wts[l], L["gate"], L["up"], L["down"], nxt,
                                          self.ws, n_experts=self.E)
                cur = nxt
                continue
            lfm.gemv_quant(ctx, L["proj"], cur, self.p)
            if self.path == "fused":
                following = self.layers[(l + 1) % len(self.layers)]
                ctx.prefetch_next(following["router"], following["norm_w"])
                lfm.moe_decode_layer(ctx, cur, self.p, L["norm_w"], self.hout, self.normed,
                                     L["router"], self.logits, None, self.ids[l], self.wts[l],
                                     L["gate"], L["up"], L["down"], nxt, self.ws,
                                     n_experts=self.E)
            else:
                lfm.router_addnorm_route(ctx, cur, self.p, L["norm_w"], self.hout, self.normed,
                                         L["router"], self.logits, None, self.ids[l],
                                         self.wts[l], self.counter)
                if self.path == "grouped":
                    lfm.moe_prefill(ctx, self.normed, self.logits, L["gate"], L["up"], L["down"],
                                    self.pws, nxt, n_experts=self.E)
                else:
                    lfm.gemv_gather_act(ctx, L["gate"], L["up"], self.normed, self.ids[l],
                                        self.act, n_experts=self.E)
                    lfm.gemv_gather_down_combine4(ctx, L["down"], self.act, self.ids[l],
                                                  self.wts[l], nxt, n_experts=self.E)
            cur = nxt
        if self.sample is None:
            lfm.gemv_head_argmax(ctx, self.head, cur, self.keys)
        else:
            lfm.gemv_quant(ctx, self.head, cur, self.head_logits)
            self.sample.encode_draw(self.head_logits, self.keys, self.sampling, self.pos)
        lfm.token_tail(ctx, self.keys, self.tokens,
                       (self.embed, self.tail_norm_w, self.x, self.tail_normed))
        if self.sample is not None:
            self.sample.encode_mark(self.tokens, self.pos)

    def status_words(self) -> list[torch.Tensor]:
        """The device status words this stack's kernels report into (the
        fused layer's sticky workspace word, the grouped GEMMs' word)."""
        words = []
        if self.ws is not None:
            words.append(self.ws[2:3])
        if self.pws is not None:
            I = self.layers[0]["gate"].out_features // self.E
            words.append(lfm.prefill_workspace_view(self.pws, self.B, self.E, self.x.shape[1],
                                                    I)["status"])
        return words

    def check(self) -> None:
        """Waits for the stream and raises McError if any kernel of the steps
        run so far reported a wait that ran out (the tokens are then invalid)."""
        for w in self.status_words():
            lfm.raise_on_status(w, f"decode stack ({self.path})")

    def read_tokens(self) -> torch.Tensor:
        """The last step's tokens on the host, after check()."""
        self.check()
        return self.tokens.cpu()

    def launches_per_step(self) -> int:
        per_layer = {"fused": 1 if self.fuse_proj else 2, "gemv": 4,
                     "grouped": 2 + lfm.MOE_PREFILL_LAUNCHES}[self.path]
        tail = 2
        if self.sampling is not None:
            s = self.sampling
            full = (s.top_k == 0 or s.top_k >= self.head.out_features) and s.top_p >= 1.0
            draw = 1 if full else 2 + 3 * ((s.top_k > 0) + (s.top_p < 1.0))
            tail = 1 + draw + 1 + 1
        return len(self.layers) * per_layer + tail
