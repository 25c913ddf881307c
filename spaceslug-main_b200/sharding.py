"""N-sharding of the int4 GEMM over the GPUs of one node.

Output columns are independent: Y[:, n] needs only W[:, n], scales[n, :] and
LoRA B[:, n].  In the reference layout a contiguous column range of W and of
the scales is one contiguous byte range (packed byte n*(K/2) + k/2, scale
n*(K/32) + k/32), so rank r uploads columns [begin, end) with no repacking
(spaceslug_q4_weights_create with col_begin/col_end) and computes its Y shard
locally.  The only exchange is the all-gather of the fp32 Y shards over
NVLink, in two forms:

* allgather_columns / ShardedGemm: NCCL all-gather (torch.distributed) into
  a rank-major [P][M][N/P] buffer, then the re-layout kernel into row-major
  [M][N]; ShardedGemm pipelines it over row bands of the GEMM.
* ShardedGemmPush: the GEMM writes its columns straight into a row-major Y
  that every peer has mapped (CUDA IPC), and copy engines push each finished
  row band into the peers' Y while the SMs compute the next band.
"""
from __future__ import annotations


def shard_columns(n: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Column range [begin, end) of `rank`; equal shards of a multiple of `align`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    per = -(-n // world)
    per = -(-per // align) * align
    begin = min(n, rank * per)
    end = min(n, begin + per)
    if end <= begin:
        raise ValueError(f"{n} columns cannot be split over {world} ranks in units of {align}")
    return begin, end


def shard_width(n: int, world: int, align: int = 8) -> int:
    per = -(-n // world)
    return -(-per // align) * align


def allgather_columns(y_shard, n_total: int, pg, stream=None):
    """All-gather column shards [M][w] of every rank into Y [M][n_total].

    Every rank passes a shard of the same width w = shard_width(n_total, P)
    (the last rank's shard is zero-padded by the caller if n_total % P != 0).
    """
    import torch
    world = pg.get_world_size()
    m, w = y_shard.shape
    buf = torch.empty((world, m, w), dtype=y_shard.dtype, device=y_shard.device)
    if y_shard.is_cuda:
        pg.all_gather_into_tensor(buf, y_shard.contiguous())
    else:  # gloo (CPU): list form
        pg.all_gather(list(buf.unbind(0)), y_shard.contiguous())
    return buf.permute(1, 0, 2).reshape(m, world * w)[:, :n_total]


def plan_bands(m: int, bands: int, align: int = 256) -> list[tuple[int, int]]:
    """Row bands [r0, r1) of an M-row GEMM for the exchange pipeline.

    The rows are cut into `align`-row tiles (whole tiles of the prefill
    kernel); at most `bands` bands get whole tiles as evenly as possible, the
    later bands the larger ones, and the last band also takes the ragged tail.
    A last band shorter than `align` rows is merged into the one before it, so
    no band of an M > 8 GEMM becomes a decode-sized (M <= 8) launch."""
    if m < 1 or bands < 1 or align < 1:
        raise ValueError("m, bands and align must be positive")
    tiles = -(-m // align)
    b = min(bands, tiles)
    base, extra = divmod(tiles, b)
    out, r0 = [], 0
    for i in range(b):
        r1 = min(m, r0 + (base + (1 if i >= b - extra else 0)) * align)
        out.append((r0, r1))
        r0 = r1
    if len(out) > 1 and out[-1][1] - out[-1][0] < align:
        out[-2:] = [(out[-2][0], out[-1][1])]
    return out


class ShardedGemm:
    """One rank's part of an N-sharded int4 GEMM whose full Y every rank needs.

    The rank's weight handle covers columns [c0, c1) of W (a contiguous byte
    range of the reference layout, spaceslug_q4_weights_create with
    col_begin / col_end).  run(x, y) computes the rank's Y shard row band by
    row band on the caller's stream.  As soon as a band is done its shard rows
    are all-gathered (NCCL through torch.distributed, on a second stream) and
    written into the caller's row-major Y by the library's re-layout kernel
    (spaceslug_shards_relayout, on a third stream), so the NVLink exchange of
    band b overlaps the GEMM of band b + 1.  When run returns, the caller's
    stream is ordered after the last re-layout.
    """

    def __init__(self, session, handle, m: int, n_total: int, dist, device, bands: int = 2, group=None) -> None:
        import torch
        self.torch, self.session, self.h, self.dist, self.group = torch, session, handle, dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.m, self.n_total, self.k = m, n_total, handle.k
        self.c0, self.c1 = shard_columns(n_total, self.world, self.rank)
        if (handle.col_begin, handle.col_end) != (self.c0, self.c1):
            raise ValueError("the weight handle does not hold this rank's column shard")
        self.width = shard_width(n_total, self.world)
        self.device = torch.device(device)
        self.bands = plan_bands(m, bands)
        self.ys = torch.zeros((m, self.width), dtype=torch.float32, device=self.device)
        self.direct = (self.c1 - self.c0) == self.width
        self.tmp = None if self.direct else torch.empty((m, self.c1 - self.c0), dtype=torch.float32,
                                                        device=self.device)
        self.gathered = torch.empty(self.world * m * self.width, dtype=torch.float32, device=self.device)
        self.comm = torch.cuda.Stream(device=self.device)
        self.post = torch.cuda.Stream(device=self.device)

    def run(self, x, y, stream=None) -> None:
        """x: device fp32 [m][k]; y: device fp32 [m][>= n_total] (row stride y.stride(0))."""
        torch = self.torch
        if x.shape != (self.m, self.k) or not x.is_contiguous() or x.dtype != torch.float32:
            raise ValueError("x must be a contiguous fp32 [m, k] tensor")
        if y.dim() != 2 or y.shape[0] != self.m or y.shape[1] < self.n_total or y.stride(1) != 1:
            raise ValueError("y must be fp32 [m, >= n_total] with unit column stride")
        s0 = stream or torch.cuda.current_stream(self.device)
        k, w, p = self.k, self.width, self.world
        for r0, r1 in self.bands:
            rows = r1 - r0
            band = self.ys[r0:r1]
            if self.direct:
                self.h.run(x.data_ptr() + 4 * r0 * k, band.data_ptr(), rows, s0.cuda_stream)
            else:
                self.h.run(x.data_ptr() + 4 * r0 * k, self.tmp[r0:r1].data_ptr(), rows, s0.cuda_stream)
                with torch.cuda.stream(s0):
                    band[:, : self.c1 - self.c0].copy_(self.tmp[r0:r1])
            done = torch.cuda.Event()
            done.record(s0)
            self.comm.wait_event(done)
            g = self.gathered[p * r0 * w: p * r1 * w].view(p * rows, w)
            with torch.cuda.stream(self.comm):
                self.dist.all_gather_into_tensor(g, band, group=self.group)
            got = torch.cuda.Event()
            got.record(self.comm)
            self.post.wait_event(got)
            self.session.shards_relayout(g.data_ptr(), y[r0:r1].data_ptr(), p, rows, w, self.n_total, y.stride(0),
                                         self.post.cuda_stream)
        fin = torch.cuda.Event()
        fin.record(self.post)
        s0.wait_event(fin)


class ShardedGemmPush:
    """The N-sharded GEMM with the exchange pushed into peer-mapped Y over NVLink.

    Every rank's full Y [m][n_total] is one device allocation, mapped into
    every other rank by CUDA IPC (spaceslug_ipc_export / spaceslug_ipc_open).
    The GEMM of each row band writes this rank's columns [c0, c1) straight
    into its own Y (spaceslug_q4_weights_run_strided, row pitch n_total), and
    as soon as the band is done its rows go to the same place in every
    peer's Y while the GEMM computes the next band.  No gather buffer and no
    re-layout.  Two engines:

    * engine="copy": one pitched copy per peer (spaceslug_copy_2d) on the
      copy engines, no SMs.  A copy engine moves a pitched copy row by row
      (~80 ns per row measured on B200), so this suits few peers.
    * engine="sm": one spaceslug_push_rows kernel per band (plain peer
      stores, each element read once and stored to every peer) on
      `push_sms` SMs that the GEMM leaves free
      (spaceslug_q4_weights_set_sm_budget) while a push runs beside it.
    * engine="epilogue": one GEMM call (spaceslug_q4_weights_run_push) whose
      epilogue stores every finished 32 x 32 block of Y to the peers as well,
      so the exchange runs tile by tile beside the next tile's main loop; no
      bands, no separate push kernel.

    Two one-element NCCL all-reduces per call fence the pushes: one before
    the first push (every rank's earlier use of its Y is done) and one after
    the last (every rank's Y is complete).  Construct and close()
    collectively on every rank.
    """

    def __init__(self, session, handle, m: int, n_total: int, dist, device, bands: int = 4, group=None,
                 engine: str = "copy", push_sms: int = 16) -> None:
        import torch
        if engine not in ("copy", "sm", "epilogue"):
            raise ValueError("engine is 'copy', 'sm' or 'epilogue'")
        self.torch, self.session, self.h, self.dist, self.group = torch, session, handle, dist, group
        self.engine = engine
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.m, self.n_total, self.k = m, n_total, handle.k
        self.c0, self.c1 = shard_columns(n_total, self.world, self.rank)
        if (handle.col_begin, handle.col_end) != (self.c0, self.c1):
            raise ValueError("the weight handle does not hold this rank's column shard")
        self.device = torch.device(device)
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.push_sms = max(1, min(int(push_sms), self.sm_count - 2))
        self.bands = plan_bands(m, 1 if engine == "epilogue" else bands)
        self.y = torch.empty((m, n_total), dtype=torch.float32, device=self.device)
        self.fence = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.comm = torch.cuda.Stream(device=self.device)
        mine = session.ipc_export(self.y.data_ptr())
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self.peers = []  # (peer rank, mapped pointer to the peer's Y, base for ipc_close)
        try:
            for r, (hb, off) in enumerate(every):
                if r != self.rank:
                    ptr, base = session.ipc_open(hb, off, self.device.index)
                    self.peers.append((r, ptr, base))
        except Exception:
            self._unmap()
            raise
        n_streams = {"copy": len(self.peers), "sm": min(1, len(self.peers)), "epilogue": 0}[engine]
        self.push_streams = [torch.cuda.Stream(device=self.device, priority=-1) for _ in range(n_streams)]

    def _unmap(self) -> None:
        for _, _, base in self.peers:
            self.session.ipc_close(base)
        self.peers = []

    def close(self) -> None:
        """Unmaps the peers' Y on every rank before any rank may free its own."""
        self.torch.cuda.synchronize(self.device)
        self._unmap()
        self.dist.barrier(group=self.group)

    def _fence(self, s0) -> None:
        torch = self.torch
        e = torch.cuda.Event()
        e.record(s0)
        self.comm.wait_event(e)
        for ps in self.push_streams:
            e = torch.cuda.Event()
            e.record(ps)
            self.comm.wait_event(e)
        with torch.cuda.stream(self.comm):
            self.dist.all_reduce(self.fence, group=self.group)

    def run(self, x, stream=None):
        """x: device fp32 [m][k].  Returns Y (this object's [m][n_total] tensor),
        complete on every rank once the caller's stream reaches this point."""
        torch = self.torch
        if x.shape != (self.m, self.k) or not x.is_contiguous() or x.dtype != torch.float32:
            raise ValueError("x must be a contiguous fp32 [m, k] tensor")
        s0 = stream or torch.cuda.current_stream(self.device)
        n, k, c0 = self.n_total, self.k, self.c0
        cols = self.c1 - self.c0
        if self.peers:
            self._fence(s0)
            start = torch.cuda.Event()
            start.record(self.comm)
            for ps in self.push_streams:
                ps.wait_event(start)
        yb = self.y.data_ptr()
        if self.engine == "epilogue":
            if self.peers:
                s0.wait_event(start)  # the GEMM's pushes start once every rank is done with its Y
            off = 4 * c0
            self.h.run_push(x.data_ptr(), yb + off, self.m, n, [ptr + off for _, ptr, _ in self.peers],
                            s0.cuda_stream)
            if self.peers:
                self._fence(s0)
                fin = torch.cuda.Event()
                fin.record(self.comm)
                s0.wait_event(fin)
            return self.y
        sm = self.engine == "sm" and bool(self.peers)
        try:
            for b, (r0, r1) in enumerate(self.bands):
                off = 4 * (r0 * n + c0)
                if sm:  # bands after the first run beside the previous band's push
                    self.h.set_sm_budget(0 if b == 0 else self.sm_count - self.push_sms)
                self.h.run_strided(x.data_ptr() + 4 * r0 * k, yb + off, r1 - r0, n, s0.cuda_stream)
                if not self.peers:
                    continue
                done = torch.cuda.Event()
                done.record(s0)
                for ps in self.push_streams:
                    ps.wait_event(done)
                if sm:
                    ps = self.push_streams[0]
                    self.session.push_rows(yb + off, [ptr + off for _, ptr, _ in self.peers], r1 - r0, cols, n,
                                           2 * self.push_sms, ps.cuda_stream)
                else:
                    for (_, ptr, _), ps in zip(self.peers, self.push_streams):
                        self.session.copy_2d(ptr + off, 4 * n, yb + off, 4 * n, 4 * cols, r1 - r0, ps.cuda_stream)
        finally:
            if sm:
                self.h.set_sm_budget(0)
        if self.peers:
            self._fence(s0)
            fin = torch.cuda.Event()
            fin.record(self.comm)
            s0.wait_event(fin)
        return self.y


# The exchange each world size uses when the caller gives no X to time
# candidates on, chosen from measurements of configs[4] (X 4096 x 8192,
# W 8192 x 28672, fp32 Y of 470 MB) on B200 boxes of this kind, each step
# timed with the L2 flushed:
#   P = 2, 4: the GEMM epilogue pushes every finished block to the peers once
#     the accumulator is back with the MMA (0.82 / 0.67 ms per step; the SM
#     push: 1.00 / 0.73 ms);
#   P = 8: banded GEMM with an SM push kernel beside it (0.776 ms on 16 SMs,
#     0.786 on 24; the epilogue push 0.788): bound by the 411 MB of Y each GPU
#     receives.
# A P not listed takes the nearest listed one below it.
EXCHANGE_BY_WORLD = {
    2: {"engine": "epilogue", "bands": 1, "push_sms": 16},
    4: {"engine": "epilogue", "bands": 1, "push_sms": 16},
    8: {"engine": "sm", "bands": 4, "push_sms": 16},
}


def choose_exchange(world: int) -> dict:
    """The exchange (engine, bands, push_sms) this library uses for `world` ranks."""
    if world < 2:
        return {"engine": "none", "bands": 1, "push_sms": 0}
    return dict(EXCHANGE_BY_WORLD[max(p for p in EXCHANGE_BY_WORLD if p <= world)])


CANDIDATES = (
    {"engine": "epilogue", "bands": 1, "push_sms": 16},
    {"engine": "sm", "bands": 4, "push_sms": 16},
    {"engine": "sm", "bands": 4, "push_sms": 24},
    {"engine": "sm", "bands": 8, "push_sms": 32},
)
_tuned: dict = {}


def autotune_exchange(session, handle, m: int, n_total: int, dist, device, x, stream=None, group=None,
                      candidates=CANDIDATES, reps: int = 3) -> dict:
    """Times each candidate exchange on this problem with every rank and returns
    the fastest (step time = max over ranks, mean of `reps` calls after one
    warm-up; ties go to the earlier candidate).  Every rank measures the same
    candidates in the same order and sees the same maxima, so every rank picks
    the same one.  The choice is cached per (world, m, n_total, k); the
    timings are in the returned dict under "tuning_ms"."""
    import torch
    world = dist.get_world_size(group)
    key = (world, m, n_total, handle.k)
    if key in _tuned:
        return dict(_tuned[key])
    dev = torch.device(device)
    s0 = stream or torch.cuda.current_stream(dev)
    times = []
    for cand in candidates:
        ex = ShardedGemmPush(session, handle, m, n_total, dist, dev, bands=cand["bands"], group=group,
                             engine=cand["engine"], push_sms=cand["push_sms"])
        try:
            ex.run(x, s0)
            evs = []
            with torch.cuda.stream(s0):
                for _ in range(reps):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(s0)
                    ex.run(x, s0)
                    b.record(s0)
                    evs.append((a, b))
            s0.synchronize()
            t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs) / reps], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            times.append(float(t.item()))
        finally:
            ex.close()
    out = pick_fastest(candidates, times)
    _tuned[key] = out
    return dict(out)


def pick_fastest(candidates, times) -> dict:
    """The candidate with the smallest time (ties to the earlier one), with
    every candidate's time under "tuning_ms"."""
    if len(candidates) != len(times) or not candidates:
        raise ValueError("one time per candidate")
    best = min(range(len(candidates)), key=lambda i: (times[i], i))
    out = dict(candidates[best])
    out["tuning_ms"] = {f"{c['engine']}_b{c['bands']}_s{c['push_sms']}": round(float(t), 4)
                        for c, t in zip(candidates, times)}
    return out


def make_sharded(session, handle, m: int, n_total: int, dist, device, group=None, tune_x=None, stream=None,
                 **override):
    """The N-sharded GEMM with the exchange for this world size: measured on
    the caller's X when tune_x is given (autotune_exchange), else the table
    choose_exchange; keyword arguments override either.  Returns a
    ShardedGemmPush; its run(x, stream) returns the full Y on every rank."""
    if tune_x is not None:
        ch = autotune_exchange(session, handle, m, n_total, dist, device, tune_x, stream=stream, group=group)
    else:
        ch = choose_exchange(dist.get_world_size(group))
    ch.update(override)
    if ch["engine"] == "none":
        raise ValueError("one rank needs no exchange: run the handle directly")
    return ShardedGemmPush(session, handle, m, n_total, dist, device, bands=ch["bands"], group=group,
                           engine=ch["engine"], push_sms=ch["push_sms"])
