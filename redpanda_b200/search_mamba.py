"""Search Mamba on the sm_100a kernels: the MARS node-evaluation surfaces.

Mirror of ``redpanda/engine/search_mamba.py`` (same heads, parameter names and
initialisation) over :class:`redpanda_b200.mamba.Mamba`.  The O(1) node step
(``eval_step``, ``evaluate_lines_fast``, ``score_branch``) runs the recurrent
step kernel; priming runs the scan with ``return_state``.
``dynamics_rollout`` (the training rollout, search_mamba.py:252-273) uses the
equivalent causal scan over the concatenated board + move tokens, so it is
differentiable through the scan kernel's analytic backward.  Checkpoint I/O
(search_mamba.py:347-383) is not part of the scan/step path and is not
mirrored; the heads keep the reference's parameter names, so a state dict that
the reference saved loads with ``load_state_dict``.
"""

import torch
import torch.nn as nn

from .graphs import StepGraph
from .mamba import Mamba, MambaConfig


class SearchMambaConfig(MambaConfig):
    """Mirrors the reference subclass (search_mamba.py:24-36).

    Like the reference, the class is not re-decorated as a dataclass, so its
    annotated defaults do not reach ``__init__``; callers pass shapes explicitly.
    """
    d_model: int = 384
    n_layer: int = 12
    d_state: int = 32
    expand: int = 2
    use_complex: bool = True
    mimo_p: int = 2
    use_bcnorm: bool = True


class SearchMamba(nn.Module):
    """Causal Mamba + value / continuation / consistency heads (search_mamba.py:39-101)."""

    def __init__(self, config: SearchMambaConfig = None, vocab_size: int = 8192,
                 eval_dim: int = 512):
        super().__init__()
        if config is None:
            config = SearchMambaConfig(vocab_size=vocab_size)
        config.bidirectional = False
        self.config = config
        self.eval_dim = eval_dim
        self.backbone = Mamba(config)
        d = config.d_model
        self.line_value_head = nn.Sequential(
            nn.Linear(d, d), nn.GELU(), nn.LayerNorm(d),
            nn.Linear(d, d // 2), nn.GELU(), nn.Linear(d // 2, 1))
        self.value_head = nn.Sequential(
            nn.Linear(d, d), nn.GELU(), nn.LayerNorm(d), nn.Linear(d, 1))
        self.continuation_head = nn.Sequential(
            nn.Linear(d, d * 2), nn.GELU(), nn.LayerNorm(d * 2),
            nn.Linear(d * 2, config.vocab_size))
        self.consistency_proj = nn.Sequential(
            nn.Linear(d, d), nn.GELU(), nn.Linear(d, eval_dim))
        self.apply(self._init_weights)
        self._node_graph = None
        self._line_graphs = {}

    def _init_weights(self, m):
        if isinstance(m, nn.Linear):
            nn.init.orthogonal_(m.weight, gain=1.0)
            if m.bias is not None:
                nn.init.constant_(m.bias, 0)

    def _device(self):
        return next(self.parameters()).device

    # -- full-sequence scoring (search_mamba.py:103-158)
    def forward(self, board_encoding, move_sequences):
        hidden = self.backbone(torch.cat([board_encoding, move_sequences], dim=-1))
        return self.line_value_head(hidden[:, -1, :]).squeeze(-1)

    def evaluate_lines(self, board_encoding, move_sequences):
        if board_encoding.dim() == 1:
            board_encoding = board_encoding.unsqueeze(0)
        return self.forward(board_encoding.expand(move_sequences.shape[0], -1), move_sequences)

    def evaluate_with_continuation(self, board_encoding, move_sequences):
        if board_encoding.dim() == 1:
            board_encoding = board_encoding.unsqueeze(0)
        full = torch.cat([board_encoding.expand(move_sequences.shape[0], -1), move_sequences], -1)
        final = self.backbone(full)[:, -1, :]
        return self.line_value_head(final).squeeze(-1), self.continuation_head(final)

    # -- O(1) cached evaluation (search_mamba.py:162-291)
    def prime_board(self, board_encoding):
        if not torch.is_tensor(board_encoding):
            board_encoding = torch.as_tensor(board_encoding, dtype=torch.long,
                                             device=self._device())
        if board_encoding.dim() == 1:
            board_encoding = board_encoding.unsqueeze(0)
        return self.backbone.prime_cache(board_encoding)

    @staticmethod
    def _expand_cache(cache, k):
        """Broadcast a B=1 cache to B=k rows (contiguous copies, as the reference)."""
        return [(h.expand(k, *h.shape[1:]).contiguous(), dbu.expand(k, *dbu.shape[1:]).contiguous())
                for h, dbu in cache]

    @torch.no_grad()
    def evaluate_lines_fast(self, board_encoding, move_sequences, lengths=None, graphed=False):
        """search_mamba.py:178-219.  ``graphed``: the K lines step through a
        captured CUDA graph of the whole backbone step (one launch per move;
        the graph for K lines is captured on first use and kept, see
        ``release_graphs``); same results up to rounding (the graph runs the
        fused step layer, the eager path the step kernel and torch's gate)."""
        device = self._device()
        _, cache = self.prime_board(board_encoding.to(device))
        K, L = move_sequences.shape
        move_sequences = move_sequences.to(device)
        hiddens = []
        if graphed:
            g = self._line_graphs.get(K)
            if g is None:
                g = self._line_graphs[K] = StepGraph(self.backbone, K)
            for (h, d), (h1, d1) in zip(g.cache, cache):   # broadcast the board's state
                h.copy_(h1.expand_as(h))
                d.copy_(d1.expand_as(d))
            for t in range(L):
                hiddens.append(g.step(move_sequences[:, t])[0].clone())
        else:
            cache = self._expand_cache(cache, K)
            for t in range(L):
                hidden, cache = self.backbone.step_(token_id=move_sequences[:, t], cache=cache)
                hiddens.append(hidden)
        hiddens = torch.stack(hiddens, dim=1)
        if lengths is not None:
            idx = (lengths.to(device).clamp(min=1) - 1).view(K, 1, 1).expand(-1, 1, hiddens.shape[-1])
            final = hiddens.gather(1, idx).squeeze(1)
        else:
            final = hiddens[:, -1, :]
        return self.line_value_head(final).squeeze(-1)

    @torch.no_grad()
    def score_branch(self, board_cache, move_sequence):
        device = self._device()
        cache = self._expand_cache(board_cache, 1)
        hidden = None
        for tok in move_sequence:
            hidden, cache = self.backbone.step_(
                token_id=torch.tensor([int(tok)], device=device), cache=cache)
        quality = self.line_value_head(hidden).squeeze(-1)
        return quality.item(), self.continuation_head(hidden).squeeze(0)

    @torch.no_grad()
    def eval_step(self, cache, move_token):
        """One O(1) node evaluation for MARS (search_mamba.py:275-291).

        Returns (value, continuation logits, new cache); ``cache`` is not modified.
        """
        tok = torch.tensor([int(move_token)], device=self._device())
        h, cache = self.backbone.step(token_id=tok, cache=cache)
        value = torch.tanh(self.value_head(h)).squeeze(-1).item()
        return value, self.continuation_head(h).squeeze(0), cache

    @torch.no_grad()
    def eval_step_graphed(self, cache, move_token):
        """``eval_step`` with the whole node step -- every layer of the backbone
        and the value and continuation heads -- replayed as one captured CUDA
        graph (:class:`redpanda_b200.graphs.StepGraph`).  Same contract: returns
        (value, continuation logits, new cache) and leaves ``cache`` unchanged;
        the new cache's tensors share one buffer, so the next call loads it with
        a single copy.  The graph is captured on first use from the current
        weights; call ``release_graphs`` after changing them."""
        g = self._node_graph
        if g is None:
            g = self._node_graph = StepGraph(
                self.backbone, 1,
                head=lambda h: (torch.tanh(self.value_head(h)).squeeze(-1),
                                self.continuation_head(h).squeeze(0)))
        g.load_(cache)
        _, value, logits = g.step(int(move_token))
        return value.item(), logits.clone(), g.snapshot()

    def release_graphs(self):
        """Drop the captured graphs (node evaluation, line batches); they are
        captured again on next use -- call after changing the weights."""
        self._node_graph = None
        self._line_graphs = {}

    def dynamics_rollout(self, board_encoding, move_tokens):
        """Training rollout (search_mamba.py:252-273) as one causal scan.

        Priming on the board and stepping through the moves is the same
        recurrence as scanning the concatenated sequence; the hidden state
        after move t is the scan output at position L_board + t.
        """
        Lb = board_encoding.shape[1]
        hidden = self.backbone(torch.cat([board_encoding, move_tokens], dim=1))[:, Lb:]
        values = torch.tanh(self.value_head(hidden)).squeeze(-1)
        return values, self.continuation_head(hidden), self.consistency_proj(hidden)
