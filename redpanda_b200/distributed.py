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
