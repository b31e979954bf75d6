"""The lockstep recurrent step of a whole Mamba stack as one CUDA graph.

A rollout (the MARS batched lines, redpanda/engine/mars_search.py:440-446) and
a search node evaluation (``SearchMamba.eval_step``,
redpanda/engine/search_mamba.py:275-291) advance the same state one token per
call through every layer: embedding, per layer RMSNorm, the in_proj / x_proj /
dt_proj GEMMs, the fused step kernels and out_proj with the residual add, then
the final norm (``Mamba.step_fused_``).  That is about ten launches per layer;
for a batch-1 node the GPU work of each is a few microseconds, so the CPU's
launch rate sets the node rate.  ``StepGraph`` records the stack once with
``torch.cuda.CUDAGraph`` and replays it as a single launch per token.

The graph reads fixed addresses: its own token buffer, its static state
(``cache``), the model's parameters and the padded step parameters cached at
capture.  So: capture after the weights are final (capture again after they
change); load a state by priming into ``cache``
(``model.prime_cache(ids, out=graph.cache)``), by ``load_`` (a copy), or by
stepping from the zero state; read ``hidden`` (and the head outputs) before the
next replay, which overwrites them.  The whole state lives in one flat buffer,
so copying a cache in or out is a single copy.
"""

import collections.abc
import numbers

import torch


class StepGraph:
    """``Mamba.step_fused_`` over every layer, captured for ``batch`` rows.

    ``head``: optional callable on the step's hidden state (B, d_model) whose
    outputs are captured too (e.g. a search's value and continuation heads);
    they are returned by :meth:`step` after the hidden state.
    """

    def __init__(self, model, batch, apply_final_norm=True, head=None, warmup=2):
        cfg = model.config
        if cfg.bidirectional:
            raise ValueError("StepGraph: the step needs a causal model")
        dev = model.embedding.weight.device
        if dev.type != "cuda":
            raise RuntimeError("StepGraph: the model must be on a CUDA device")
        n_layer, d, n = len(model.layers), cfg.d_inner, cfg.d_state
        self.model = model
        self.batch = batch
        self._per = batch * d * n
        self.flat = torch.zeros(n_layer * 2 * self._per, device=dev, dtype=torch.float32)
        self.cache = self._views(self.flat)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self._pinned = None     # host staging of per-row ids (step)

        def run(cache):
            h, _ = model.step_fused_(token_id=self.tokens, cache=cache,
                                     apply_final_norm=apply_final_norm)
            extra = head(h) if head is not None else ()
            return (h, *extra) if isinstance(extra, tuple) else (h, extra)

        # warm-up on a scratch state (cuBLAS handles, the library's kernel
        # attributes and the padded step parameters are set up here, outside
        # the capture) so the caller's state is not advanced
        scratch = self._views(self.flat.clone())
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(warmup):
                run(scratch)
        torch.cuda.current_stream(dev).wait_stream(side)
        del scratch
        # thread-local capture: CUDA calls from other threads of the process
        # (NCCL's watchdog in a multi-GPU job) do not invalidate it
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.outputs = run(self.cache)
        self.hidden = self.outputs[0]

    def _views(self, flat):
        """(h, dBu) views of each layer's slice of a flat state buffer."""
        d, n = self.model.config.d_inner, self.model.config.d_state
        per, b = self._per, self.batch
        return [(flat[(2 * i) * per:(2 * i + 1) * per].view(b, d, n),
                 flat[(2 * i + 1) * per:(2 * i + 2) * per].view(b, d, n))
                for i in range(len(self.model.layers))]

    def load_(self, cache):
        """Copy a cache ((h, dBu) per layer, ``batch`` rows) into the static state."""
        src = getattr(cache, "flat", None)
        if src is not None and src.numel() == self.flat.numel():
            self.flat.copy_(src)
            return
        if len(cache) != len(self.cache):
            raise ValueError("load_: one (h, dBu) entry per layer")
        dst = [t for pair in self.cache for t in pair]
        torch._foreach_copy_(dst, [t for pair in cache for t in pair[:2]])

    def snapshot(self):
        """A copy of the static state as a new cache (one copy of the flat buffer)."""
        return FlatCache(self.flat.clone(), self._views, len(self.cache))

    def reset_(self):
        """Zero state (the reference's ``init_cache``: no prefix)."""
        self.flat.zero_()

    def step(self, token_id):
        """Advance the static state by one token per row; returns the captured
        outputs (hidden state first), valid until the next call.

        ``token_id``: one id for every row (a Python or numpy integer: written
        by a fill kernel, with no host-to-device copy and so no wait for the
        GPU), or one per row as a tensor or sequence (a CUDA tensor is copied
        on the device; host ids go through a pinned buffer, asynchronously)."""
        if isinstance(token_id, numbers.Integral):
            self.tokens.fill_(int(token_id))
        elif torch.is_tensor(token_id) and token_id.is_cuda:
            self.tokens.copy_(token_id.reshape(-1))
        else:
            tok = torch.as_tensor(token_id).reshape(-1)
            if self._pinned is None:
                self._pinned = torch.empty(self.batch, dtype=torch.long, pin_memory=True)
                self._pinned_done = torch.cuda.Event()
            self._pinned_done.synchronize()   # the last copy out of it has run
            self._pinned.copy_(tok.expand(self.batch) if tok.numel() == 1 else tok)
            self.tokens.copy_(self._pinned, non_blocking=True)
            self._pinned_done.record()
        self.graph.replay()
        return self.outputs


class FlatCache(collections.abc.Sequence):
    """A cache, (h, dBu) per layer, whose tensors are views of one buffer,
    ``flat``.  The per-layer views are made on first access: a search that only
    hands the cache back to :meth:`StepGraph.load_` (one copy of ``flat``)
    never pays for them."""

    def __init__(self, flat, views, n):
        self.flat = flat
        self._make = views
        self._n = n
        self._views = None

    def __len__(self):
        return self._n

    def __getitem__(self, i):
        if self._views is None:
            self._views = self._make(self.flat)
        return self._views[i]


def _main():
    """Time the config-3 backbone's step graph: ``python -m redpanda_b200.graphs
    --batch 1``.  Reference initialisation, random move ids; prints the CUDA-event
    time per replayed step."""
    import argparse
    from .mamba import Mamba, Mamba3Block, MambaConfig
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=str, default="1", help="comma-separated batch sizes")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--small", type=int, default=Mamba3Block.small_step_max_batch,
                    help="Mamba3Block.small_step_max_batch (0: cuBLAS projections)")
    ap.add_argument("--steps", type=int, default=20)
    args = ap.parse_args()
    torch.manual_seed(0)
    cfg = MambaConfig(d_model=512, n_layer=args.layers, d_state=32, n_track_state=8, mimo_p=2,
                      vocab_size=8192)
    model = Mamba(cfg).cuda().eval()
    Mamba3Block.small_step_max_batch = args.small
    for batch in (int(b) for b in args.batch.split(",")):
        g = StepGraph(model, batch)
        moves = torch.randint(0, cfg.vocab_size, (batch,), device="cuda")
        for _ in range(3):
            g.step(moves)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g.step(moves)
        e1.record()
        torch.cuda.synchronize()
        print(f"batch {batch}: {e0.elapsed_time(e1) / args.steps * 1e3:.1f} us per step "
              f"(small_step_max_batch {args.small})", flush=True)


if __name__ == "__main__":
    _main()
