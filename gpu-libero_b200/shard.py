"""World shards across GPUs and the observation gather to rank 0.

Worlds are independent, so a multi-GPU job is one process per GPU, each
owning the contiguous world range [rank * W, (rank + 1) * W) with seeds
drawn by global world index (scene.initial_state / scene.actions take the
shard's `world_offset`); the physics step has no collective.  The one data
exchange is the optional gather of every rank's observation slab
([W, nobs], the step kernel's `obs` output) so that rank 0 holds the whole
batch: an all-gather over NCCL (NVLink / NVSwitch) issued on a side stream
right after a control step, overlapped with the next one.
"""
import torch
import torch.distributed as dist


def shard_offset(rank, worlds_per_rank):
    """Global index of the first world of `rank`."""
    return rank * worlds_per_rank


def all_gather_into(out, inp, group=None):
    """out[r * W:(r + 1) * W] = inp of rank r, on every rank."""
    n = dist.get_world_size(group)
    if out.shape[0] != n * inp.shape[0] or out.shape[1:] != inp.shape[1:]:
        raise ValueError('gather buffer has shape %s, expected %s' % (tuple(out.shape), (n * inp.shape[0],) +
                                                                    tuple(inp.shape[1:])))
    if dist.get_backend(group) == 'nccl':
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.chunk(n)), inp, group=group)


class ObservationGather:
    """Gather of `runtime.buffers['obs']` from every rank into `self.out`.

    `launch()` is called on the stream that enqueued a control step: it
    snapshots the slab (so the next step may overwrite it) and all-gathers the
    snapshot on a side stream.  `wait()` makes the current stream wait for the
    latest gather.  Every rank must call `launch()` the same number of times.
    """

    def __init__(self, runtime, group=None):
        self.group = group
        self.src = runtime.buffers['obs']
        n = dist.get_world_size(group)
        self.stage = torch.empty_like(self.src)
        self.out = torch.empty((n * self.src.shape[0],) + tuple(self.src.shape[1:]), dtype=self.src.dtype,
                               device=self.src.device)
        self.cuda = self.src.is_cuda
        self.stream = torch.cuda.Stream(self.src.device) if self.cuda else None
        self.done = None
        self.count = 0

    def launch(self):
        if not self.cuda:
            self.stage.copy_(self.src)
            all_gather_into(self.out, self.stage, self.group)
            self.count += 1
            return
        current = torch.cuda.current_stream(self.src.device)
        if self.done is not None:
            current.wait_event(self.done)  # the previous gather still reads the snapshot
        self.stage.copy_(self.src)
        self.stream.wait_stream(current)
        with torch.cuda.stream(self.stream):
            all_gather_into(self.out, self.stage, self.group)
            self.done = torch.cuda.Event()
            self.done.record(self.stream)
        self.count += 1

    def wait(self):
        if self.cuda and self.done is not None:
            torch.cuda.current_stream(self.src.device).wait_event(self.done)

    def bytes_per_launch(self):
        return self.out.numel() * self.out.element_size()
