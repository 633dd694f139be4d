"""Tensor-parallel sharding of the decoder for single-tree latency (T = 2, 4 or 8 GPUs, one process per GPU).

Rank r of T holds:
  * q heads [r * hq/T, (r+1) * hq/T) and KV heads [r * hk/T, (r+1) * hk/T) of every layer (column-parallel QKV;
    a query head's KV head h // (hq/hk) stays on the same rank), and the K/V pools of its KV heads;
  * the matching columns of the O projection (row-parallel): its partial [n, hidden] output is summed over ranks
    (all-reduce) before the post-attention norms;
  * intermediate slice [r * F/T, (r+1) * F/T) of the gate and up projections (column-parallel) and the matching
    columns of the down projection (row-parallel, all-reduced before the post-MLP norms);
  * the embedding, norms, layer scalars and the label head whole (replicated; every rank computes the same
    probabilities).
The tree plan is deterministic, so every rank plans the same steps on the host.
"""
from .checkpoint import PREFIX, layer_geometry


def shard_config(top, world):
    """The per-rank config: local head counts and intermediate size."""
    cfg = dict(top['text_config'])
    hq = cfg['num_attention_heads']
    for key in ('num_attention_heads', 'num_key_value_heads', 'num_global_key_value_heads', 'intermediate_size'):
        if cfg[key] % world:
            raise ValueError(f'{key} = {cfg[key]} is not divisible by {world} ranks')
    if (cfg['intermediate_size'] // world) % 128:
        raise ValueError('each rank needs a multiple of 128 intermediate rows (GeGLU tile layout)')
    for kind in ('sliding_attention', 'full_attention'):
        hk, _ = layer_geometry(cfg, kind)
        if (hq // world) % (hk // world) and (hk // world) % (hq // world):
            raise ValueError('query heads per KV head must stay on one rank')
    cfg['num_attention_heads'] = hq // world
    cfg['num_key_value_heads'] //= world
    cfg['num_global_key_value_heads'] //= world
    cfg['intermediate_size'] //= world
    return dict(top, text_config=cfg)


def shard_getter(top, get, rank, world):
    """`get(key)` for rank `rank`: the full tensor's shard (a contiguous copy), replicated tensors unchanged."""
    cfg = top['text_config']
    hq, F = cfg['num_attention_heads'], cfg['intermediate_size']

    def rows(t, n, width=1):
        per = n // world
        return t[rank * per * width:(rank + 1) * per * width].contiguous()

    def cols(t, n, width=1):
        per = n // world
        return t[:, rank * per * width:(rank + 1) * per * width].contiguous()

    def g(key):
        t = get(key)
        if not key.startswith(PREFIX + 'layers.'):
            return t
        i = int(key[len(PREFIX + 'layers.'):].split('.')[0])
        kind = cfg['layer_types'][i]
        hk, d = layer_geometry(cfg, kind)
        if key.endswith('self_attn.q_proj.weight'):
            return rows(t, hq, d)
        if key.endswith(('self_attn.k_proj.weight', 'self_attn.v_proj.weight')):
            return rows(t, hk, d)
        if key.endswith('self_attn.o_proj.weight'):
            return cols(t, hq, d)
        if key.endswith(('mlp.gate_proj.weight', 'mlp.up_proj.weight')):
            return rows(t, F)
        if key.endswith('mlp.down_proj.weight'):
            return cols(t, F)
        return t
    return g


# ---- peer-memory exchange (the all-reduce of the row-parallel projections, fused with the epilogues) ------------

MAX_RANKS = 8
BLOCK = 128


def exchange_layout(world, hidden, max_rows):
    """Byte layout of one rank's exchange allocation: its partial rows of a row-parallel projection (read by the row
    blocks' owners), the x and h rows of a whole step, and the two per-block counter arrays. Every region starts on
    a 256-byte boundary."""
    max_blocks = max(1, -(-max_rows // BLOCK))
    rows = max_blocks * BLOCK * hidden * 2
    sizes = dict(part=rows, x=rows, h=rows, partials=max_blocks * 8, rows=max_blocks * 8)
    off, layout = 0, {}
    for name in ('part', 'x', 'h', 'partials', 'rows'):
        layout[name] = (off, sizes[name])
        off += -(-sizes[name] // 256) * 256
    return dict(max_blocks=max_blocks, regions=layout, nbytes=off)


def owner(block, world):
    """The rank that reduces row block `block`."""
    return block % world


def partial_target(sites, world, hidden):
    """A block's partial-column counter after `sites` reductions: every rank delivers 4 x hidden columns per block
    per site (4 epilogue warps of 32 rows, each counting the columns of every tile it stored)."""
    return sites * world * 4 * hidden


def row_target(sites):
    """A block's row counter after `sites` reductions: its owner pushes 128 rows to every rank per site."""
    return sites * BLOCK


def gather_handles(group, handle):
    """Every rank's IPC handle bytes, in rank order (a collective over `group`)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


class PassProtocol:
    """Host-side agreement of a tensor-parallel group around every pass over peer memory.

    The exchange kernels wait on counters that other ranks advance, and give up after a bounded time (device codes
    0x104 / 0x105). Two host rules keep that bound from firing, or from leaving the group out of step, when the ranks'
    hosts do not start a pass together (planning a larger tree, a request arriving on one rank later, a pause):
      * `begin()` before a pass launches anything: a barrier over the group, so no rank's kernels start waiting on
        a peer whose host has not reached the pass yet;
      * `agree(code)` after the pass: the largest device error code over the group, so every rank sees a failure any
        rank saw, and `recover(clear)` then runs on all of them: wait for the GPU, barrier, zero the counters
        (`clear`), barrier. The next pass then starts every counter from zero again (the host's cumulative targets
        restart with `sites` = 0)."""

    def __init__(self, group, device=None):
        import torch.distributed as dist
        self.group = group
        self.device = device if dist.get_backend(group) == 'nccl' else None

    def begin(self):
        import torch.distributed as dist
        dist.barrier(group=self.group)

    def agree(self, code):
        import torch
        import torch.distributed as dist
        t = torch.tensor([int(code)], dtype=torch.int64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return int(t.item())

    def recover(self, clear):
        import torch
        import torch.distributed as dist
        if self.device is not None:
            torch.cuda.synchronize(self.device)  # every wait still running ends by its own bound
        dist.barrier(group=self.group)
        clear()
        if self.device is not None:
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)


class PeerExchange:
    """This rank's exchange buffers, mapped into every peer (CUDA IPC), and the `morj_peer_t` that describes them.

    Collective: every rank of `group` constructs it with the same arguments. `sites` counts the reductions run so
    far; every rank runs the same sequence, so the cumulative counter targets agree."""

    def __init__(self, group, hidden, max_rows, device):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _native as nat
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f'peer exchange supports up to {MAX_RANKS} ranks')
        lay = exchange_layout(self.world, hidden, max_rows)
        self.hidden, self.max_rows = hidden, lay['max_blocks'] * BLOCK
        self.buf = torch.zeros(lay['nbytes'], dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)  # counters are zero before any peer can signal them
        handle = ctypes.create_string_buffer(nat.IPC_HANDLE_BYTES)
        nat.call('morj_ipc_export', self.buf.data_ptr(), handle)
        handles = gather_handles(group, handle.raw)
        self.bases, self._opened = [], []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.buf.data_ptr())
                continue
            ptr = ctypes.c_void_p()
            nat.call('morj_ipc_import', hb, ctypes.byref(ptr))
            self.bases.append(ptr.value)
            self._opened.append((ptr.value, hb))
        d = nat.PeerDesc()
        d.world, d.rank, d.max_blocks, d.hidden = self.world, self.rank, lay['max_blocks'], hidden
        for r, base in enumerate(self.bases):
            for name in ('part', 'x', 'h', 'partials', 'rows'):
                getattr(d, name)[r] = base + lay['regions'][name][0]
        self.desc = d
        self.regions = lay['regions']
        self.sites = 0
        self.protocol = PassProtocol(group, device)
        dist.barrier(group=group)

    def begin_pass(self):
        """Before a pass launches anything (see `PassProtocol.begin`)."""
        self.protocol.begin()

    def end_pass(self, code):
        """After a pass: the group's largest device error code; on a failure anywhere, every rank zeroes its counters
        and restarts the site count (see `PassProtocol`)."""
        code = self.protocol.agree(code)
        if code:
            self.protocol.recover(self._clear_counters)
        return code

    def _clear_counters(self):
        for name in ('partials', 'rows'):
            off, size = self.regions[name]
            self.buf[off:off + size].zero_()
        self.sites = 0

    def rows_view(self, name, n):
        """This rank's x or h rows [n, hidden] (BF16) inside the exchange allocation."""
        import torch
        off, _ = self.regions[name]
        return self.buf[off:off + n * self.hidden * 2].view(torch.bfloat16).view(n, self.hidden)

    def close(self):
        from . import _native as nat
        for ptr, hb in self._opened:
            nat.call('morj_ipc_close', ptr, hb)
        self._opened = []
