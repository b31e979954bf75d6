"""Data-parallel plumbing for the scan: batch sharding and one bucketed all-reduce.

The scan and the step never exchange activations between rows, so a batch is
split evenly across ranks (one process per GPU) and only parameter gradients
cross the interconnect.  :class:`ScanGradAllReducer` packs the gradients of the
scan parameters of every ``Mamba3Block`` -- ``A_log_mag``, ``A_phase`` (or
``A_log``), ``track_theta``, ``dt_proj.bias``, ``b_norm.weight``,
``c_norm.weight`` -- into one flat fp32 bucket, all-reduces it once (NCCL over
NVLink on GPUs, gloo on CPU), averages, and unpacks.  Other parameters can be
included with ``extra``; a full data-parallel trainer passes all of them.

The reference trains on a single GPU and has no distributed code; this module
is new plumbing around the kernels, not part of the kernels.
"""

import datetime

import torch
import torch.distributed as dist

SCAN_PARAM_SUFFIXES = ("A_log_mag", "A_phase", "A_log", "track_theta", "dt_proj.bias",
                       "b_norm.weight", "c_norm.weight")


def shard_rows(n_rows, rank, world):
    """[start, stop) of the rows rank ``rank`` owns (sizes differ by at most 1)."""
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def scan_parameters(module):
    """(name, parameter) pairs of the scan parameters of ``module``, in a fixed order."""
    return [(n, p) for n, p in module.named_parameters()
            if p.requires_grad and n.endswith(SCAN_PARAM_SUFFIXES)]


class ScanGradAllReducer:
    """One all-reduce of a fixed set of parameter gradients per step.

    Every rank must build it over the same model (same parameter order) and call
    :meth:`synchronize` at the same point of every step.  Gradients that are
    ``None`` on a rank contribute zeros.
    """

    def __init__(self, module=None, params=None, extra=(), group=None, average=True):
        named = list(params) if params is not None else scan_parameters(module)
        named += list(extra)
        if not named:
            raise ValueError("no parameters to reduce")
        self.names = [n for n, _ in named]
        self.params = [p for _, p in named]
        self.group = group
        self.average = average
        self.numel = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.bucket = torch.zeros(self.numel, dtype=torch.float32, device=dev)

    def synchronize(self):
        """Pack, all-reduce (sum, then / world size), unpack into ``.grad``."""
        off = 0
        for p in self.params:
            n = p.numel()
            if p.grad is None:
                self.bucket[off:off + n].zero_()
            else:
                self.bucket[off:off + n].copy_(p.grad.reshape(-1))
            off += n
        dist.all_reduce(self.bucket, op=dist.ReduceOp.SUM, group=self.group)
        if self.average:
            self.bucket.div_(dist.get_world_size(self.group))
        off = 0
        for p in self.params:
            n = p.numel()
            g = self.bucket[off:off + n].view_as(p).to(p.dtype)
            if p.grad is None:
                p.grad = g.clone()
            else:
                p.grad.copy_(g)
            off += n
        return self.bucket


class OverlappedGradAllReducer:
    """Bucketed all-reduce of parameter gradients, launched during the backward.

    Parameters are grouped into buckets of about ``bucket_bytes`` in reverse
    registration order (roughly the order the backward produces their
    gradients: last layer first).  A post-accumulate-grad hook on every
    parameter counts down its bucket; when the bucket's last gradient has
    landed, the bucket is packed and its all-reduce is started asynchronously
    (NCCL runs it on its own stream behind the compute already queued), so it
    overlaps the rest of the backward.  :meth:`finish` waits for the buckets,
    averages and unpacks them into ``.grad``; buckets that were never completed
    (a parameter without a gradient this step) are reduced there, with zeros
    standing in for missing gradients, so every rank issues the same
    collectives in the same order.

    With gradient accumulation, call :meth:`arm` before the backward of the
    last micro-batch only; the hooks do nothing while disarmed.
    """

    def __init__(self, module=None, params=None, bucket_bytes=8 << 20, group=None,
                 average=True):
        plist = list(params) if params is not None else \
            [p for p in module.parameters() if p.requires_grad]
        if not plist:
            raise ValueError("no parameters to reduce")
        self.group = group
        self.average = average
        self.buckets = []
        cur, size = [], 0
        for p in reversed(plist):
            cur.append(p)
            size += p.numel() * 4
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self.bucket_of = {}
        for bi, b in enumerate(self.buckets):
            for p in b:
                self.bucket_of[p] = bi
                p.register_post_accumulate_grad_hook(self._hook)
        self.armed = False
        self._reset()

    def _reset(self):
        self.pending = [len(b) for b in self.buckets]
        self.started = {}

    def arm(self):
        self._reset()
        self.armed = True

    def _pack(self, bi):
        return torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1)
                          .to(torch.float32) for p in self.buckets[bi]])

    def _start(self, bi):
        flat = self._pack(bi)
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self.started[bi] = (flat, work)

    def _hook(self, p):
        if not self.armed:
            return
        bi = self.bucket_of[p]
        self.pending[bi] -= 1
        # buckets start in index order, so every rank issues the same sequence
        # of collectives even when its backward finishes buckets in another order
        if self.pending[bi] == 0:
            nxt = len(self.started)
            while nxt < len(self.buckets) and self.pending[nxt] == 0:
                self._start(nxt)
                nxt += 1

    def finish(self):
        """Wait for every bucket, average, and write the results into ``.grad``."""
        for bi in range(len(self.buckets)):
            if bi not in self.started:
                self._start(bi)
        world = dist.get_world_size(self.group)
        for bi, b in enumerate(self.buckets):
            flat, work = self.started[bi]
            work.wait()
            if self.average:
                flat.div_(world)
            off = 0
            for p in b:
                n = p.numel()
                g = flat[off:off + n].view_as(p).to(p.dtype)
                if p.grad is None:
                    p.grad = g.clone()
                else:
                    p.grad.copy_(g)
                off += n
        self.armed = False
        self._reset()


def init_from_env(backend=None, timeout_s=300):
    """init_process_group from torchrun's environment with a bounded timeout.

    Returns (rank, world_size, local_rank).  A single process without the
    environment variables is world size 1 and initialises nothing.
    """
    import os
    if "WORLD_SIZE" not in os.environ or int(os.environ["WORLD_SIZE"]) == 1:
        return 0, 1, int(os.environ.get("LOCAL_RANK", "0"))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    local = int(os.environ.get("LOCAL_RANK", "0"))
    kwargs = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return dist.get_rank(), dist.get_world_size(), local
