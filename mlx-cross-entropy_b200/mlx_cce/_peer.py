"""Exchange buffers of the vocabulary-sharded backward (NVLink peer memory).

The cross-rank sum of grad_e runs inside the library's own kernels
(``cce_backward_peer``): the last grad_e GEMM of every rank stores its output
tiles straight into the buffer of the rank that owns those rows, the owners sum
them, and every rank copies the summed rows back (csrc/peer.cuh describes the
buffer and the flags).  This module owns the host side: one buffer per
(process group, device), allocated by the library as a driver virtual-memory
allocation; its POSIX file descriptor is sent to every other rank over an
abstract-namespace Unix datagram socket (SCM_RIGHTS: descriptors cannot travel
through the process group's own tensors), and the other ranks' buffers are
mapped into this process with access for this rank's device only.  The
buffers grow when a call needs more room (every rank grows at the same call,
since all ranks pass the same N and D) and live until ``release_all()`` or
process exit.

The reference has no multi-device code; this is the build's own plumbing for
the multi-GPU rows of the benchmark.
"""

from __future__ import annotations

import ctypes
import os
import random
import socket
import struct
import threading

import torch
import torch.distributed as dist

from . import _ext

# Bound of each wait on another rank inside the exchange kernels; after it the
# call's grad_e is invalid and cce_device_status reports the rank that never came.
DEFAULT_WAIT_MS = 10_000

_groups: dict = {}


class PeerGroup:
    """Exchange buffers of one process group on one CUDA device."""

    def __init__(self, group, device: torch.device):
        self.group = group
        self.device = device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _ext.CCE_PEER_MAX_WORLD:
            raise ValueError(f"the peer exchange supports at most {_ext.CCE_PEER_MAX_WORLD} ranks, "
                             f"got {self.world}")
        self.bytes = 0
        self.own = None
        self.opened: list = []
        self.struct = None

    def ensure(self, nbytes: int) -> _ext.CcePeerGroup:
        """The group's CcePeerGroup with buffers of at least ``nbytes`` (collective)."""
        if nbytes <= self.bytes:
            return self.struct
        self._release()
        own, fd = ctypes.c_void_p(), ctypes.c_int(-1)
        with torch.cuda.device(self.device):
            _ext._check(_ext.lib.cce_peer_buffer_alloc(nbytes, ctypes.byref(own), ctypes.byref(fd)),
                        "cce_peer_buffer_alloc")
        self.own = own.value
        try:
            fds = self._exchange_fds(fd.value)
        finally:
            os.close(fd.value)
        bases = [0] * self.world
        bases[self.rank] = self.own
        try:
            for r, rfd in fds.items():
                ptr = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _ext._check(_ext.lib.cce_peer_buffer_open(rfd, nbytes, ctypes.byref(ptr)),
                                "cce_peer_buffer_open")
                self.opened.append(ptr.value)
                bases[r] = ptr.value
        finally:
            for rfd in fds.values():
                os.close(rfd)
        st = _ext.CcePeerGroup()
        st.rank, st.world = self.rank, self.world
        st.wait_limit_ns = int(float(os.environ.get("CCE_PEER_WAIT_MS", DEFAULT_WAIT_MS)) * 1e6)
        st.bytes = nbytes
        for r, b in enumerate(bases):
            st.bases[r] = b
        self.bytes = nbytes
        self.struct = st
        # every rank has mapped every buffer before any kernel writes into one
        dist.barrier(group=self.group)
        return st

    def _exchange_fds(self, fd: int) -> dict:
        """Send this rank's descriptor to every other rank; return {rank: their descriptor}.

        One abstract-namespace datagram socket per rank, named after a token
        drawn by the group; a thread receives while the main thread sends, so
        no sender blocks on a full receive queue.
        """
        mine = torch.tensor([random.getrandbits(62)], dtype=torch.int64, device=self.device)
        every = torch.empty(self.world, dtype=torch.int64, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=self.group)
        token = int(every[0].item())
        name = lambda r: b"\0cce-peer-%d-%d-%d" % (os.getuid(), token, r)
        sock = socket.socket(socket.AF_UNIX, socket.SOCK_DGRAM)
        sock.bind(name(self.rank))
        got: dict = {}
        errors: list = []

        def receive():
            try:
                for _ in range(self.world - 1):
                    msg, fds, _flags, _addr = socket.recv_fds(sock, 16, 1)
                    if len(msg) < 4 or len(fds) != 1:
                        raise RuntimeError("malformed descriptor message from a peer rank")
                    got[struct.unpack("i", msg[:4])[0]] = fds[0]
            except Exception as exc:  # reported below
                errors.append(exc)

        th = threading.Thread(target=receive, daemon=True)
        th.start()
        try:
            dist.barrier(group=self.group)   # every rank's socket exists
            for r in range(self.world):
                if r != self.rank:
                    # (socket.send_fds takes no destination address for datagrams)
                    sock.sendmsg([struct.pack("i", self.rank)],
                                 [(socket.SOL_SOCKET, socket.SCM_RIGHTS, struct.pack("i", fd))], 0, name(r))
            th.join(timeout=60)
            if th.is_alive() or errors or len(got) != self.world - 1:
                raise RuntimeError(f"exchange-buffer descriptors from {len(got)} of {self.world - 1} ranks "
                                   f"arrived ({errors[0] if errors else 'timeout'})")
        finally:
            sock.close()
        dist.barrier(group=self.group)
        return got

    def _release(self):
        """Unmap the other ranks' buffers and free this rank's (collective)."""
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)   # no exchange kernel of this rank still runs
        dist.barrier(group=self.group)        # ... nor of any other rank
        with torch.cuda.device(self.device):
            for p in self.opened:
                _ext._check(_ext.lib.cce_peer_buffer_close(p), "cce_peer_buffer_close")
            dist.barrier(group=self.group)    # every rank has unmapped this rank's buffer
            _ext._check(_ext.lib.cce_peer_buffer_free(self.own), "cce_peer_buffer_free")
        self.own, self.opened, self.bytes, self.struct = None, [], 0, None


def buffer_bytes(N: int, D: int, world: int, out_dtype: torch.dtype) -> int:
    return int(_ext.lib.cce_peer_buffer_bytes(N, D, world, _ext.dtype_code(out_dtype, "cce_peer_buffer_bytes")))


def group_for(group, device: torch.device, N: int, D: int, out_dtype: torch.dtype) -> _ext.CcePeerGroup:
    """The CcePeerGroup for a backward of N x D rows on this group (collective when it grows)."""
    key = (id(group), device.index)
    pg = _groups.get(key)
    if pg is None:
        pg = _groups[key] = PeerGroup(group, device)
    return pg.ensure(buffer_bytes(N, D, pg.world, out_dtype))


def release_all():
    """Free every exchange buffer of this process (collective over each group)."""
    for key in list(_groups):
        _groups.pop(key)._release()
