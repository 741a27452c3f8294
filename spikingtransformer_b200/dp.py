"""Data-parallel gradient synchronisation for the training step.

The reference trains on one GPU (``train_spikeformer.py:2``); the training
benchmark runs the same step data-parallel, one process per GPU, and sums the
gradients over NCCL in bf16.  ``BucketedGradReducer`` does that inside a CUDA
graph as well as eagerly:

* every trainable parameter's gradient is a view into one flat fp32 buffer
  (the optimizer reads the views, nothing is copied back);
* the parameters are grouped into buckets of contiguous ranges of that
  buffer, from the last registered parameter backwards, which is roughly the
  order in which the backward finishes them;
* when the last gradient of a bucket has been accumulated (a
  post-accumulate-grad hook), the bucket is cast to bf16, all-reduced (sum)
  over the process group and written back divided by the world size, on a
  side stream, so the transfer overlaps the rest of the backward;
* ``finish()`` launches the buckets whose parameters received no gradient in
  this backward (every rank has the same ones, so the collectives stay in the
  same order on every rank) and makes the current stream wait for the side
  stream.

Under CUDA graph capture the hooks run while the backward is captured, so the
graph holds the casts and collectives at the points where their buckets
complete.  A graph that holds collectives must be released before the
process group is destroyed.
"""

import torch
import torch.distributed as dist


class BucketedGradReducer:
    def __init__(self, params, bucket_elems=4 << 20, comm_dtype=torch.bfloat16, group=None):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dev = self.params[0].device
        self.group = group
        self.world = dist.get_world_size(group)
        total = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(total, dtype=torch.float32, device=dev)
        offsets = []
        off = 0
        for p in self.params:
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            offsets.append(off)
            off += p.numel()
        # buckets of whole parameters, from the last one backwards
        self.buckets = []  # (start, end, member count)
        bucket_of = [0] * len(self.params)
        members, n = [], 0
        for i in reversed(range(len(self.params))):
            members.append(i)
            n += self.params[i].numel()
            if n >= bucket_elems or i == 0:
                lo = min(offsets[j] for j in members)
                hi = max(offsets[j] + self.params[j].numel() for j in members)
                for j in members:
                    bucket_of[j] = len(self.buckets)
                self.buckets.append((lo, hi, len(members)))
                members, n = [], 0
        self.comm = None if comm_dtype == torch.float32 else torch.empty(total, dtype=comm_dtype, device=dev)
        self.stream = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self._remaining = [b[2] for b in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._hooks = [p.register_post_accumulate_grad_hook(self._make_hook(bucket_of[i]))
                       for i, p in enumerate(self.params)]

    def _make_hook(self, b):
        def hook(_param):
            self._remaining[b] -= 1
            if self._remaining[b] == 0:
                self._launch(b)
        return hook

    def begin(self):
        """Zero the gradients (the views stay in place) and arm the hooks for one
        backward."""
        self.flat.zero_()
        self._remaining = [b[2] for b in self.buckets]
        self._launched = [False] * len(self.buckets)

    def _launch(self, b):
        if self._launched[b]:
            return
        self._launched[b] = True
        if self.stream is None:
            self._reduce(b)
            return
        self.stream.wait_stream(torch.cuda.current_stream(self.flat.device))
        with torch.cuda.stream(self.stream):
            self._reduce(b)

    def _reduce(self, b):
        lo, hi, _ = self.buckets[b]
        g = self.flat[lo:hi]
        if self.comm is None:
            dist.all_reduce(g, group=self.group)
            g.div_(self.world)
        else:
            c = self.comm[lo:hi]
            c.copy_(g)
            dist.all_reduce(c, group=self.group)
            g.copy_(c).div_(self.world)

    def finish(self):
        """Launch the buckets the backward did not complete and join the side
        stream; after this the gradients hold the average over the ranks."""
        for b in range(len(self.buckets)):
            if not self._launched[b]:
                self._launch(b)
        if self.stream is not None:
            torch.cuda.current_stream(self.flat.device).wait_stream(self.stream)

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
