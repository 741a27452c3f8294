"""Forward passes over batches held in pinned host memory.

``stream_forward`` runs a module over a sequence of host batches with the
copies overlapped with the compute.  Three streams take part:

- the caller's current stream runs the forward of batch i;
- a host-to-device stream copies batch i+1 into the other of two device slots
  while batch i computes, and waits for batch i-1's forward to finish with
  that slot first;
- a device-to-host stream copies the result of batch i into its pinned host
  buffer as soon as the forward of batch i ends.

Every batch still crosses PCIe both ways.  Only the waiting is hidden.
"""

import torch

__all__ = ["stream_forward"]


def _check_pinned(t, what):
    if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
        raise ValueError("%s must be a CPU tensor" % what)
    if not t.is_pinned():
        raise ValueError("%s must be in pinned host memory (tensor.pin_memory())" % what)


def stream_forward(fn, host_inputs, host_outputs, device=None):
    """Run ``fn`` over host batches and copy every result back to the host.

    Parameters
    ----------
    fn : callable
        ``fn(*device_tensors) -> device tensor``.  It runs on the current
        stream of ``device``.
    host_inputs : sequence of tuples of pinned CPU tensors
        Batch i is ``host_inputs[i]``.  Every batch has the shapes and dtypes
        of the first.
    host_outputs : sequence of pinned CPU tensors
        The result of batch i is copied into ``host_outputs[i]``, which must
        match its shape and dtype.  One buffer may appear at several
        positions; the copies into it run in order.
    device : torch.device, optional
        Defaults to the current CUDA device.

    Every copy and forward is enqueued before this returns.  The current
    stream waits for the last result copy, so a synchronize of that stream,
    or an event recorded on it, covers all the work.
    """
    n = len(host_inputs)
    if len(host_outputs) != n:
        raise ValueError("host_outputs has %d entries for %d batches" % (len(host_outputs), n))
    if n == 0:
        return
    first = tuple(host_inputs[0])
    for i, batch in enumerate(host_inputs):
        batch = tuple(batch)
        if len(batch) != len(first):
            raise ValueError("batch %d has %d tensors, batch 0 has %d" % (i, len(batch), len(first)))
        for j, (t, t0) in enumerate(zip(batch, first)):
            if not isinstance(t, torch.Tensor) or t.shape != t0.shape or t.dtype != t0.dtype:
                raise ValueError("host_inputs[%d][%d] differs in shape or dtype from batch 0" % (i, j))
    for i, batch in enumerate(host_inputs):
        for j, t in enumerate(batch):
            _check_pinned(t, "host_inputs[%d][%d]" % (i, j))
    for i, t in enumerate(host_outputs):
        _check_pinned(t, "host_outputs[%d]" % i)
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)

    comp = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    # the slots are allocated on the compute stream, which also reads them
    slots = [[torch.empty(t.shape, dtype=t.dtype, device=device) for t in first] for _ in range(2)]
    h2d.wait_stream(comp)
    d2h.wait_stream(comp)
    ready = [None] * n
    done = [None] * n
    copied = [None] * n

    def copy_in(i):
        with torch.cuda.stream(h2d):
            if i >= 2:
                # the slot's previous batch has been consumed, and its result
                # copied out (the result may alias the slot)
                h2d.wait_event(done[i - 2])
                h2d.wait_event(copied[i - 2])
            for dst, src in zip(slots[i % 2], host_inputs[i]):
                dst.copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            ready[i] = ev

    copy_in(0)
    for i in range(n):
        if i + 1 < n:
            copy_in(i + 1)
        comp.wait_event(ready[i])
        out = fn(*slots[i % 2])
        if not isinstance(out, torch.Tensor) or out.device != device:
            raise ValueError("fn must return a tensor on %s" % device)
        if out.shape != host_outputs[i].shape or out.dtype != host_outputs[i].dtype:
            raise ValueError("result %d has shape %s %s, host_outputs[%d] has %s %s"
                             % (i, tuple(out.shape), out.dtype, i, tuple(host_outputs[i].shape),
                                host_outputs[i].dtype))
        ev = torch.cuda.Event()
        ev.record(comp)
        done[i] = ev
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev)
            host_outputs[i].copy_(out, non_blocking=True)
            copied[i] = torch.cuda.Event()
            copied[i].record(d2h)
        out.record_stream(d2h)  # keep the result's memory until its copy ends
    comp.wait_stream(d2h)
    for s in slots:
        for t in s:
            t.record_stream(h2d)
