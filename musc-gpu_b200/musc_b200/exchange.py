"""Copy-engine transport of the multi-GPU pool scoring (one process per GPU, one node).

``pipeline.score_pool`` exchanges three things per bank between the ranks:

* the centring statistics of every rank's rows (column sums, smallest row norm), so
  that every rank centres its bank rows on the same pool mean before the split (a few
  KB, copied on the compute stream);
* the bank planes: every rank preps the bank of its own query images and needs the
  whole pool's bank (an all-gather);
* the screen tables: every rank screens its share of the symmetric tiles into tables
  blocked by the rows' owners, and each owner needs its block from every rank (an
  all-to-all).

With NCCL these collectives need SMs, and they cannot start while the persistent
screening GEMM holds every SM -- so they run between the GEMMs instead of under them.
Here they are peer copies on copy engines: every rank maps its peers' buffers through
CUDA IPC once, and per bank each rank's copy streams pull the peers' planes and table
blocks as soon as the peers signal them ready.  Readiness and release are 32-bit
counters in device memory, written with stream-ordered writes into the peer's flags and
awaited with stream-ordered waits on one's own flags, so no host synchronisation and no
SM time is involved.  A mapped peer pointer is only ever a copy source: no kernel and no
library routine reads a peer's memory.

Flags of rank r (``[world][6]`` uint32, written by the peers, row = the writer):
``BANK_READY`` (the writer's bank k is prepared), ``BANK_TAKEN`` (the writer has copied
r's bank k, so r may reuse the buffer), ``SCREEN_READY``, ``SCREEN_TAKEN``,
``SUMS_READY``, ``SUMS_TAKEN`` (the same for the centring statistics).  The value is
the exchange's bank counter, which only grows (across calls too), so a wait for
``>= v`` never confuses banks.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib, ops

BANK_READY, BANK_TAKEN, SCREEN_READY, SCREEN_TAKEN, SUMS_READY, SUMS_TAKEN = range(6)
N_FLAGS = 6
FLAGS_SLOT, STATS_SLOT = 6, 7   # positions of the flags and of stats[0] among the shared buffers


def _vp(x: int) -> ctypes.c_void_p:
    return ctypes.c_void_p(int(x))


class PeerExchange:
    """Buffers and IPC mappings of one pool shape on one rank (create collectively)."""

    def __init__(self, group, device, n_images: int, patches: int, channels: int, n_copy_streams: int = 4):
        import torch.distributed as dist
        from .pipeline import shard_range
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.n_images, self.p, self.c = n_images, patches, channels
        _, _, self.per = shard_range(n_images, self.world, 0)
        self.rows = n_images * patches
        self.local_rows = self.per * patches
        self.bank_rows = self.world * self.local_rows
        self.rpb = self.local_rows
        dev = self.device
        lib = _lib.lib()
        with torch.cuda.device(dev):
            # read by the peers
            self.local_bank = [ops.empty_bank(self.local_rows, channels, dev) for _ in range(2)]
            self.screens = [ops.screen_table(self.rows, patches, self.rpb, dev, min_blocks=self.world)
                            for _ in range(2)]
            self.flags = torch.zeros(self.world, N_FLAGS, dtype=torch.int32, device=dev)
            self.stats = [torch.zeros(channels + 1, dtype=torch.float64, device=dev) for _ in range(2)]
            # filled by this rank's copies
            self.full_bank = [ops.empty_bank(self.bank_rows, channels, dev) for _ in range(3)]
            self.stats_all = [torch.empty(self.world, channels + 1, dtype=torch.float64, device=dev)
                              for _ in range(2)]
            self.recv = [(torch.empty(self.world, n_images, self.rpb, dtype=torch.int64, device=dev),
                          torch.empty(self.world, n_images, self.rpb, dtype=torch.int32, device=dev))
                         for _ in range(2)]
            self.copy_streams = [torch.cuda.Stream(dev) for _ in range(max(1, n_copy_streams))]
            torch.cuda.synchronize(dev)
        # IPC handles of the buffers the peers read, exchanged once
        shared = [self.local_bank[0], self.local_bank[1], self.screens[0][0], self.screens[0][1],
                  self.screens[1][0], self.screens[1][1], self.flags, self.stats[0], self.stats[1]]
        mine = []
        for t in shared:
            h = (ctypes.c_ubyte * 64)()
            off = ctypes.c_size_t(0)
            with torch.cuda.device(dev):
                _lib.check(lib.musc_b200_ipc_get(_vp(t.data_ptr()), h, ctypes.byref(off)), 'musc_b200_ipc_get')
            mine.append((bytes(h), off.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self._bases = []
        self.peer = {}   # peer rank -> list of mapped pointers (same order as `shared`)
        with torch.cuda.device(dev):
            for s in range(self.world):
                if s == self.rank:
                    continue
                ptrs = []
                for handle, off in everyone[s]:
                    base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
                    hb = (ctypes.c_ubyte * 64).from_buffer_copy(handle)
                    _lib.check(lib.musc_b200_ipc_open(hb, off, ctypes.byref(base), ctypes.byref(ptr)),
                               'musc_b200_ipc_open')
                    self._bases.append(base.value)
                    ptrs.append(ptr.value)
                self.peer[s] = ptrs
        # plane offsets (bytes) of a rank's local bank and of the pool bank
        self._local_offs = self._plane_offsets(self.local_rows)
        self._full_offs = self._plane_offsets(self.bank_rows)
        self._plane_bytes = [self.local_rows * channels * 2] * 2 + [self.local_rows * 4] * 3
        self.counter = 0          # banks exchanged so far (monotonic)
        self._refined = {}        # bank counter -> event after the bank's last use of full_bank / recv
        dist.barrier(group=group)

    def _plane_offsets(self, rows: int) -> list[int]:
        offs = (ctypes.c_size_t * 5)()
        _lib.check(_lib.lib().musc_b200_bank_layout(rows, self.c, offs), 'musc_b200_bank_layout')
        return list(offs)

    def matches(self, n_images: int, patches: int, channels: int, world: int) -> bool:
        return (n_images, patches, channels, world) == (self.n_images, self.p, self.c, self.world)

    # ------------------------------------------------------------------ flag helpers
    def _my_flag(self, writer: int, kind: int) -> ctypes.c_void_p:
        return _vp(self.flags.data_ptr() + (writer * N_FLAGS + kind) * 4)

    def _peer_flag(self, peer: int, kind: int) -> ctypes.c_void_p:
        # this rank's row in the peer's flags
        return _vp(self.peer[peer][FLAGS_SLOT] + (self.rank * N_FLAGS + kind) * 4)

    def _signal_peers(self, kind: int, value: int, stream) -> None:
        lib = _lib.lib()
        for s in self.peer:
            _lib.check(lib.musc_b200_stream_signal(self._peer_flag(s, kind), value, _vp(stream.cuda_stream)),
                       'musc_b200_stream_signal')

    def _wait(self, writer: int, kind: int, value: int, stream) -> None:
        _lib.check(_lib.lib().musc_b200_stream_wait(self._my_flag(writer, kind), value, _vp(stream.cuda_stream)),
                   'musc_b200_stream_wait')

    def _copy(self, dst: int, src: int, nbytes: int, stream) -> None:
        _lib.check(_lib.lib().musc_b200_copy_async(_vp(dst), _vp(src), nbytes, _vp(stream.cuda_stream)),
                   'musc_b200_copy_async')

    def _stream_of(self, peer: int):
        return self.copy_streams[peer % len(self.copy_streams)]

    # ------------------------------------------------------------------ per bank
    def begin_bank(self) -> int:
        """Counter value of the next bank (1, 2, ...)."""
        self.counter += 1
        return self.counter

    def center(self, v: int, compute, z_local: torch.Tensor, kernels) -> torch.Tensor:
        """Centring statistics of bank ``v``: this rank reduces its rows ``z_local`` on
        ``compute``, signals the peers and copies every rank's statistics (the compute stream
        waits for each peer's).  Returns the ``(world, C + 1)`` fp64 statistics for the
        centred prep."""
        if v > 2:
            for s in self.peer:
                self._wait(s, SUMS_TAKEN, v - 2, compute)
        mine = self.stats[v % 2]
        kernels.center_stats(z_local, out=mine)
        self._signal_peers(SUMS_READY, v, compute)
        out = self.stats_all[v % 2]
        nb = (self.c + 1) * 8
        for s in range(self.world):
            if s == self.rank:
                src = mine.data_ptr()
            else:
                self._wait(s, SUMS_READY, v, compute)
                src = self.peer[s][STATS_SLOT + v % 2]
            self._copy(out.data_ptr() + s * nb, src, nb, compute)
            if s != self.rank:
                _lib.check(_lib.lib().musc_b200_stream_signal(self._peer_flag(s, SUMS_TAKEN), v,
                                                              _vp(compute.cuda_stream)), 'musc_b200_stream_signal')
        return out

    def local_bank_for(self, v: int, compute) -> torch.Tensor:
        """This rank's bank buffer for bank ``v``, once every peer has copied bank ``v - 2``
        out of it (the compute stream waits)."""
        if v > 2:
            for s in self.peer:
                self._wait(s, BANK_TAKEN, v - 2, compute)
        return self.local_bank[v % 2]

    def gather(self, v: int, compute):
        """After this rank prepared bank ``v`` into ``local_bank_for(v)`` on ``compute``: signal
        the peers and pull their banks into the pool bank on the copy streams.  Returns
        ``(pool bank, events)``: whoever reads the pool bank waits for the events first."""
        full = self.full_bank[v % 3]
        ready = torch.cuda.Event()
        ready.record(compute)
        self._signal_peers(BANK_READY, v, compute)
        free = self._refined.get(v - 3)
        done = []
        for s in range(self.world):
            st = self._stream_of(s)
            if free is not None:
                st.wait_event(free)
            if s == self.rank:
                st.wait_event(ready)
                src = self.local_bank[v % 2].data_ptr()
            else:
                self._wait(s, BANK_READY, v, st)
                src = self.peer[s][v % 2]
            for lo, fo, nb in zip(self._local_offs, self._full_offs, self._plane_bytes):
                self._copy(full.data_ptr() + fo + s * nb, src + lo, nb, st)
            if s != self.rank:
                _lib.check(_lib.lib().musc_b200_stream_signal(self._peer_flag(s, BANK_TAKEN), v,
                                                              _vp(st.cuda_stream)), 'musc_b200_stream_signal')
            ev = torch.cuda.Event()
            ev.record(st)
            done.append(ev)
        return full, done

    def screen_for(self, v: int, compute):
        """This rank's screen tables for bank ``v``, once every peer has copied its block of
        bank ``v - 2`` (the compute stream waits)."""
        if v > 2:
            for s in self.peer:
                self._wait(s, SCREEN_TAKEN, v - 2, compute)
        return self.screens[v % 2]

    def exchange(self, v: int, compute):
        """After this rank screened bank ``v`` on ``compute``: signal the peers and pull this
        rank's block of every rank's tables.  Returns ``(k1, m2, events)``; the refinement
        waits for ``events`` and then :meth:`release` records its end."""
        k1, m2 = self.recv[v % 2]
        ready = torch.cuda.Event()
        ready.record(compute)
        self._signal_peers(SCREEN_READY, v, compute)
        free = self._refined.get(v - 2)
        block_k = self.n_images * self.rpb * 8
        block_m = self.n_images * self.rpb * 4
        done = []
        for s in range(self.world):
            st = self._stream_of(s)
            if free is not None:
                st.wait_event(free)
            if s == self.rank:
                st.wait_event(ready)
                src_k, src_m = self.screens[v % 2][0].data_ptr(), self.screens[v % 2][1].data_ptr()
            else:
                self._wait(s, SCREEN_READY, v, st)
                src_k, src_m = self.peer[s][2 + 2 * (v % 2)], self.peer[s][3 + 2 * (v % 2)]
            self._copy(k1.data_ptr() + s * block_k, src_k + self.rank * block_k, block_k, st)
            self._copy(m2.data_ptr() + s * block_m, src_m + self.rank * block_m, block_m, st)
            if s != self.rank:
                _lib.check(_lib.lib().musc_b200_stream_signal(self._peer_flag(s, SCREEN_TAKEN), v,
                                                              _vp(st.cuda_stream)), 'musc_b200_stream_signal')
            ev = torch.cuda.Event()
            ev.record(st)
            done.append(ev)
        return k1, m2, done

    def release(self, v: int, compute) -> None:
        """Bank ``v``'s pool bank and received tables are no longer read after this point of
        ``compute``."""
        ev = torch.cuda.Event()
        ev.record(compute)
        self._refined[v] = ev
        for old in [k for k in self._refined if k < v - 3]:
            del self._refined[old]

    def close(self) -> None:
        """Wait for everything, unmap the peers' buffers (collective: every rank calls it)."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for b in self._bases:
                _lib.check(_lib.lib().musc_b200_ipc_close(_vp(b)), 'musc_b200_ipc_close')
        self._bases = []
        self.peer = {}
