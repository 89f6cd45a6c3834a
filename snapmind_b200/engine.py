"""Greedy generation with the decode step captured in a CUDA graph.

The reference engine runs prefill and then one eager forward per token
(snapmind/engine/generate.py:108-133, snapmind/engine/decode.py:9-26), which at
batch 1 is bound by host launch overhead: hundreds of small launches per token.
``GraphDecoder`` keeps the same flow for a model whose attention layers are
``gqa_paged`` over one ``"paged"`` cache:

* the prompt is prefilled eagerly (block tables grow on the host, in the
  reference's order);
* the blocks of all decode steps are taken up front, in the order the
  per-token stores would take them (``PagedKVCache.begin_device_steps``), and
  the slot / length / position / token of the running step live in device
  tensors;
* one decode step (model forward, greedy argmax, counter updates) runs once
  as a warm-up on a side stream, is captured into a ``torch.cuda.CUDAGraph`` and
  replayed for the remaining steps: every launch of a step, the cache's append
  and decode kernels included, becomes one graph launch.

The generated ids equal an eager run's; the cache ends in the same state.

``BatchedGraphDecoder`` is the many-sequence form (the reference engine holds
one sequence): B prompts of one length are prefilled into a ``PagedKVPool``,
then every decode step grows all B sequences on the device
(``snapmind_kv_reserve``), appends their K/V rows and runs one batched paged
decode per layer — captured once and replayed, like ``GraphDecoder``.
"""
from __future__ import annotations

import torch

from snapmind_b200.kv_cache.paged import PagedKVCache
from snapmind_b200.paged_pool import PagedKVPool


class GraphDecoder:
    def __init__(self, model: torch.nn.Module, cache: PagedKVCache, use_graph: bool = True):
        self.model, self.cache, self.use_graph = model, cache, use_graph
        self.views = cache.layer_dicts()
        self._graph: torch.cuda.CUDAGraph | None = None
        self._steps_left = 0

    # ------------------------------------------------------------------ parts
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> None:
        """Run the prompt (1-D token ids) and pick the first generated token."""
        dev = self.cache.device
        self.model.eval()
        logits = self.model(prompt.reshape(1, -1).to(dev), kv_cache=self.views)[0, -1]
        self.tok = logits.argmax(-1).reshape(1, 1).clone()
        self.pos = torch.full((1,), prompt.numel(), dtype=torch.long, device=dev)

    @torch.no_grad()
    def begin(self, n_steps: int) -> None:
        """Reserve ``n_steps`` decode steps; ids are collected in ``self.ids``."""
        dev = self.cache.device
        self.ids = torch.empty(n_steps + 1, dtype=torch.long, device=dev)
        self.ids[0] = self.tok.reshape(())
        self.idx = torch.ones((1,), dtype=torch.long, device=dev)
        self.cache.begin_device_steps(n_steps)
        self._steps_total = n_steps
        self._steps_left = n_steps
        self._graph = None

    def _step(self) -> None:
        logits = self.model(self.tok, kv_cache=self.views, position_ids=self.pos)[0, -1]
        self.tok.copy_(logits.argmax(-1).reshape(1, 1))
        self.ids.index_copy_(0, self.idx, self.tok.reshape(1))
        self.cache.advance_device_step()
        self.pos.add_(1)
        self.idx.add_(1)

    @torch.no_grad()
    def step(self, n: int = 1) -> None:
        """Run ``n`` decode steps: the first eagerly (warm-up), then by graph replay."""
        for _ in range(n):
            if self._steps_left <= 0:
                raise RuntimeError("GraphDecoder: no decode steps left")
            if self._graph is None and (not self.use_graph or self._steps_left == self._steps_total):
                side = torch.cuda.Stream(self.cache.device)
                side.wait_stream(torch.cuda.current_stream(self.cache.device))
                with torch.cuda.stream(side):
                    self._step()
                torch.cuda.current_stream(self.cache.device).wait_stream(side)
                if self.use_graph and self._steps_left > 1:
                    self._graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(self._graph):  # recorded, not run
                        self._step()
            elif self._graph is not None:
                self._graph.replay()
            else:
                self._step()
            self._steps_left -= 1

    @torch.no_grad()
    def finish(self) -> list[int]:
        """End the device steps and return the generated ids."""
        if self._steps_left:
            raise RuntimeError(f"GraphDecoder: {self._steps_left} decode steps not run")
        self._graph = None
        self.cache.end_device_steps(self._steps_total)
        self.cache.check_device_errors()
        return self.ids.tolist()

    # ----------------------------------------------------------------- whole
    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, n_tokens: int) -> list[int]:
        """Greedy ids: the prefill's token, then ``n_tokens - 1`` decode steps."""
        self.prefill(prompt)
        if n_tokens <= 1:
            return [int(self.tok.item())][:n_tokens]
        self.begin(n_tokens - 1)
        self.step(n_tokens - 1)
        return self.finish()


class BatchedGraphDecoder:
    def __init__(self, model: torch.nn.Module, pool: PagedKVPool, batch: int, use_graph: bool = True):
        self.model, self.pool, self.batch, self.use_graph = model, pool, batch, use_graph
        self.views = pool.layer_views(batch)
        self._graph: torch.cuda.CUDAGraph | None = None
        self._steps_left = 0

    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor) -> None:
        """``prompts``: token ids ``[B, T]`` (one length for all sequences)."""
        dev = self.pool.device
        b, t = prompts.shape
        if b != self.batch:
            raise ValueError(f"BatchedGraphDecoder: {b} prompts for a batch of {self.batch}")
        self.model.eval()
        self.pool.reserve(t, batch=b)
        logits = self.model(prompts.to(dev), kv_cache=self.views)[:, -1]
        self.tok = logits.argmax(-1).reshape(b, 1).clone()
        self.pos = torch.full((b,), t, dtype=torch.long, device=dev)

    @torch.no_grad()
    def begin(self, n_steps: int) -> None:
        pool, b = self.pool, self.batch
        if pool.blocks_needed(n_steps, b) > pool._host_free:
            raise RuntimeError("PagedKVCache: out of blocks")
        cap = int(pool.host_lens[:b].max()) + n_steps
        if (cap + pool.block_size - 1) // pool.block_size > pool.max_blocks_per_seq:
            raise ValueError("BatchedGraphDecoder: sequences would outgrow their block table rows")
        for view in self.views.values():
            view.capacity = cap  # one split plan for every step
        self.ids = torch.empty((n_steps + 1, b), dtype=torch.long, device=pool.device)
        self.ids[0] = self.tok.reshape(b)
        self.idx = torch.ones((1,), dtype=torch.long, device=pool.device)
        self._steps_total = self._steps_left = n_steps
        self._graph = None

    def _step(self) -> None:
        self.pool.reserve_device(1, self.batch)
        logits = self.model(self.tok, kv_cache=self.views, position_ids=self.pos)[:, -1]
        self.tok.copy_(logits.argmax(-1).reshape(self.batch, 1))
        self.ids.index_copy_(0, self.idx, self.tok.reshape(1, self.batch))
        self.pos.add_(1)
        self.idx.add_(1)

    @torch.no_grad()
    def step(self, n: int = 1) -> None:
        dev = self.pool.device
        for _ in range(n):
            if self._steps_left <= 0:
                raise RuntimeError("BatchedGraphDecoder: no decode steps left")
            if self._graph is None and (not self.use_graph or self._steps_left == self._steps_total):
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    self._step()
                torch.cuda.current_stream(dev).wait_stream(side)
                if self.use_graph and self._steps_left > 1:
                    self._graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(self._graph):  # recorded, not run
                        self._step()
            elif self._graph is not None:
                self._graph.replay()
            else:
                self._step()
            self._steps_left -= 1

    @torch.no_grad()
    def finish(self) -> list[list[int]]:
        """Account the steps on the host and return each sequence's ids."""
        if self._steps_left:
            raise RuntimeError(f"BatchedGraphDecoder: {self._steps_left} decode steps not run")
        self._graph = None
        self.pool.account_host(self._steps_total, self.batch)
        for view in self.views.values():
            view.capacity = None
        self.pool.check()
        return self.ids.t().tolist()

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, n_tokens: int) -> list[list[int]]:
        self.prefill(prompts)
        if n_tokens <= 1:
            return self.tok.reshape(-1, 1)[:, :n_tokens].tolist()
        self.begin(n_tokens - 1)
        self.step(n_tokens - 1)
        return self.finish()
