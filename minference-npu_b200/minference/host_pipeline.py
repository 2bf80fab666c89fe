"""Layer attention with q/k/v in pinned host memory, transfers overlapped.

For prefill with the inputs offloaded to the host (long contexts whose
q/k/v do not stay resident on the GPU), the PCIe copies dominate a layer:
at 64K tokens and 32 heads, q/k/v are 1.2 GB in and the output 0.4 GB out,
against ~16 ms of attention.  Run one after another, the three add up.  This
module cuts the layer's heads into chunks and pipelines them over three
streams:

    copy-in stream :  H2D(chunk 0) H2D(chunk 1) H2D(chunk 2) ...
    caller's stream:              attn(chunk 0) attn(chunk 1) ...
    copy-out stream:                            D2H(chunk 0)  D2H(chunk 1) ...

Each chunk's attention waits for its own inputs only, and each copy-out
waits for its own attention.  PCIe is full duplex, so the layer takes about
as long as the larger of the inbound transfer and the attention.

The attention of a chunk is the package's per-pattern op (the same call the
patched HF forward makes for a group of heads), so results are identical to
running the ops on device-resident inputs.
"""

from __future__ import annotations

import torch

from .modules.minference_forward import _run_pattern

__all__ = ["layer_attention_from_host"]

_streams: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}
_buffers: dict[tuple, tuple[torch.Tensor, ...]] = {}


def _side_streams(dev: torch.device):
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _streams:
        _streams[idx] = (torch.cuda.Stream(device=idx), torch.cuda.Stream(device=idx))
    return _streams[idx]


def layer_attention_from_host(q_host: torch.Tensor, k_host: torch.Tensor, v_host: torch.Tensor,
                              out_host: torch.Tensor, groups, device: torch.device,
                              chunk_heads: int = 2) -> None:
    """Attention of one layer from host inputs into a host output.

    q_host, k_host, v_host: pinned CPU tensors ``[B, H, S, D]`` (BNSD,
    contiguous).  out_host: pinned CPU tensor ``[B, H, S, D]`` receiving the
    output.  groups: ``[(key, heads)]`` as produced by
    ``minference.modules.minference_forward.group_heads`` (key = pattern type
    and parameters, heads = head indices).  Every group's heads are processed
    in chunks of `chunk_heads` contiguous heads.

    The work is queued on the caller's current stream (attention) and two
    side streams (copies); the caller's stream waits for the last copy-out,
    so synchronising it (or reading out_host after torch.cuda.synchronize())
    sees the complete output.  Device buffers are cached per shape; calls on
    one device must not overlap."""
    if not (q_host.is_pinned() and k_host.is_pinned() and v_host.is_pinned()
            and out_host.is_pinned()):
        raise ValueError("q/k/v/out must be pinned host tensors")
    if q_host.dim() != 4 or q_host.shape != k_host.shape or q_host.shape != v_host.shape \
            or out_host.shape != q_host.shape:
        raise ValueError("q/k/v/out must share one [B, H, S, D] shape")
    dev = torch.device(device)
    key = (dev, tuple(q_host.shape), q_host.dtype)
    if key not in _buffers:
        _buffers[key] = tuple(torch.empty(q_host.shape, dtype=q_host.dtype, device=dev)
                              for _ in range(4))
    dq, dk, dv, do = _buffers[key]
    copy_in, copy_out = _side_streams(dev)
    main = torch.cuda.current_stream(dev)

    # Expensive groups first: a chunk's attention then overlaps the transfers
    # of the cheaper chunks behind it, and the pipeline ends on short work.
    cost = {"vertical_and_slash": 0, "dense": 0, "block_sparse": 1, "stream_llm": 2}
    groups = sorted(groups, key=lambda g: cost.get(g[0][0], 3))
    chunks = []
    for gkey, heads in groups:
        heads = list(heads)
        i = 0
        while i < len(heads):
            j = i + 1
            while j < len(heads) and j - i < chunk_heads and heads[j] == heads[j - 1] + 1:
                j += 1
            chunks.append((gkey, slice(heads[i], heads[j - 1] + 1)))
            i = j

    # The previous call's kernels and copies on these buffers are done before
    # this call's copies overwrite them.
    copy_in.wait_stream(main)
    copy_out.wait_stream(main)
    done_in, done_attn = [], []
    with torch.cuda.stream(copy_in):
        for _, sl in chunks:
            dq[:, sl].copy_(q_host[:, sl], non_blocking=True)
            dk[:, sl].copy_(k_host[:, sl], non_blocking=True)
            dv[:, sl].copy_(v_host[:, sl], non_blocking=True)
            e = torch.cuda.Event()
            e.record(copy_in)
            done_in.append(e)
    for (gkey, sl), e_in in zip(chunks, done_in):
        main.wait_event(e_in)
        _run_pattern(gkey, dq[:, sl], dk[:, sl], dv[:, sl], out=do[:, sl])
        e = torch.cuda.Event()
        e.record(main)
        done_attn.append(e)
    with torch.cuda.stream(copy_out):
        for (_, sl), e_attn in zip(chunks, done_attn):
            copy_out.wait_event(e_attn)
            out_host[:, sl].copy_(do[:, sl], non_blocking=True)
    main.wait_stream(copy_out)
