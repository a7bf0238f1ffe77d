"""Rank-0 -> follower command channel for tensor-parallel engines.

Every TP rank runs the same ``ModelRunner`` call in the same order; rank 0
decides what to run (the scheduler lives there) and tells the followers.  The
reference does this with pickled commands in a 64 MiB POSIX shared-memory
segment guarded by ``mp.Event`` objects (``nano_vllm_uno/engine/model_runner.py:154-255``).

Here the channel is one shared-memory slot with a fixed binary layout and
spin-then-sleep polling, so a decode step costs a few microseconds of host
time on every rank instead of a pickle plus a TCP broadcast:

* header (one cache line each): message sequence number, payload length,
  writer pid, then one acknowledgement word and pid per rank;
* ``run`` commands are packed with numpy: one int64 row of fixed fields per
  sequence, the page tables as one int32 vector, prompt tokens only for
  prefill, and the sampling parameters only when they changed;
* any other command (``exit``, ``reseed``, timing hooks) is pickled.

Followers rebuild light ``Sequence`` objects whose token list is a
length-plus-last-token stand-in (``TokenTail``): a decode step never copies a
request's history.  The writer waits for every follower to acknowledge the
previous message before it overwrites the slot; readers and the writer check
each other's pids while they wait, so a dead rank surfaces as an exception
instead of a hang.
"""

from __future__ import annotations

import os
import pickle
import time
from multiprocessing import resource_tracker, shared_memory

import numpy as np

from uno_b200.engine.sequence import Sequence, SequenceStatus, new_decode_stats

_LINE = 64  # bytes per header word (own cache line)
_MAX_RANKS = 64
_HDR = _LINE * (3 + 2 * _MAX_RANKS)
_DEFAULT_BYTES = 64 << 20


def channel_bytes(env=None) -> int:
    """Payload capacity of the command channel: ``INFERENCE_ENGINE_SHM_SIZE`` bytes when set (the
    reference engine's knob for large prefill batches, ``nano_vllm_uno/engine/model_runner.py:160``),
    else 64 MiB."""
    env = os.environ if env is None else env
    raw = env.get("INFERENCE_ENGINE_SHM_SIZE")
    if raw is None or not raw.strip():
        return _DEFAULT_BYTES
    size = int(raw)
    if size < 4096:
        raise ValueError(f"INFERENCE_ENGINE_SHM_SIZE={size} is below the 4096-byte minimum")
    return size

MSG_PICKLE = 1
MSG_RUN = 2

_FIELDS = 10  # seq_id, status, last_token, num_tokens, num_prompt, num_cached, max_completion, has_seed, seed, n_pages


class TokenTail:
    """Token list stand-in for follower ranks: its length and its last token."""

    __slots__ = ("n", "last")

    def __init__(self, n: int, last: int):
        self.n = int(n)
        self.last = int(last)

    def __len__(self) -> int:
        return self.n

    def __getitem__(self, i):
        if isinstance(i, int) and (i == -1 or i == self.n - 1):
            return self.last
        raise IndexError("a follower rank holds only the last token of a sequence")

    def extend(self, tokens) -> None:
        for t in tokens:
            self.n += 1
            self.last = int(t)


def _pid_alive(pid: int) -> bool:
    if pid <= 0:
        return True
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


class CommandChannel:
    """Single-slot broadcast channel in host shared memory (one writer, N-1 readers)."""

    def __init__(self, name: str | None, rank: int, world: int, size: int = _DEFAULT_BYTES,
                 timeout_s: float = 600.0):
        if world > _MAX_RANKS:
            raise ValueError(f"at most {_MAX_RANKS} ranks")
        self.rank, self.world, self.timeout_s = rank, world, float(timeout_s)
        if name is None:
            self.shm = shared_memory.SharedMemory(create=True, size=_HDR + size)
            self.owner = True
        else:
            self.shm = shared_memory.SharedMemory(name=name, create=False)
            self.owner = False
            try:  # the writer owns the segment's lifetime
                resource_tracker.unregister(self.shm._name, "shared_memory")
            except Exception:  # pragma: no cover - tracker differences across Python versions
                pass
        buf = self.shm.buf
        self._words = np.ndarray((3 + 2 * _MAX_RANKS, _LINE // 8), dtype=np.int64, buffer=buf[:_HDR])
        self.payload = buf[_HDR:]
        self.capacity = len(self.payload)
        if self.owner:
            self._words[:] = 0
            self._words[2, 0] = os.getpid()
        else:
            self._words[3 + rank, 0] = 0
        self._words[3 + _MAX_RANKS + rank, 0] = os.getpid()
        self.seen = 0

    @property
    def name(self) -> str:
        return self.shm.name

    # ------------------------------------------------------------ words
    def _seq(self) -> int:
        return int(self._words[0, 0])

    def _ack(self, r: int) -> int:
        return int(self._words[3 + r, 0])

    def _pid(self, r: int) -> int:
        return int(self._words[3 + _MAX_RANKS + r, 0])

    # ------------------------------------------------------------- wait
    def _wait(self, ready, who: str, peers) -> None:
        if ready():
            return
        t0 = time.perf_counter()
        spins = 0
        last_check = t0
        while not ready():
            spins += 1
            if spins > 2000:
                time.sleep(0 if spins < 20000 else 50e-6)
            now = time.perf_counter()
            if now - last_check > 0.5:
                last_check = now
                for r in peers:
                    if not _pid_alive(self._pid(r)):
                        raise RuntimeError(f"TP rank {r} exited while rank {self.rank} waited for {who}")
                if self.timeout_s and now - t0 > self.timeout_s:
                    raise TimeoutError(f"rank {self.rank}: no {who} within {self.timeout_s:.0f}s")

    # ----------------------------------------------------------- writer
    def begin_write(self) -> memoryview:
        """Wait until every reader consumed the previous message; return the payload buffer."""
        seq = self._seq()
        readers = range(1, self.world)
        self._wait(lambda: all(self._ack(r) >= seq for r in readers), "acknowledgements", readers)
        return self.payload

    def commit(self, nbytes: int) -> None:
        if nbytes > self.capacity:
            raise ValueError(f"command of {nbytes} bytes exceeds the {self.capacity}-byte channel "
                             "(raise INFERENCE_ENGINE_SHM_SIZE or lower max_num_seqs)")
        self._words[1, 0] = nbytes
        self._words[0, 0] = self._seq() + 1  # published last: readers see a complete payload

    # ----------------------------------------------------------- reader
    def read(self) -> bytes:
        target = self.seen + 1
        self._wait(lambda: self._seq() >= target, "a command from rank 0", [0])
        n = int(self._words[1, 0])
        data = bytes(self.payload[:n])
        self.seen = target
        self._words[3 + self.rank, 0] = target
        return data

    def close(self) -> None:
        self._words = None
        self.payload = None
        try:
            self.shm.close()
        except BufferError:  # pragma: no cover - a view is still alive
            pass
        if self.owner:
            try:
                self.shm.unlink()
            except FileNotFoundError:  # pragma: no cover
                pass


# ------------------------------------------------------------------ encoding
def _i64(v: int) -> int:
    v = int(v) & 0xFFFFFFFFFFFFFFFF
    return v - (1 << 64) if v >= (1 << 63) else v


class RunEncoder:
    """Packs ``run(seqs, is_prefill, sp)`` into the channel (rank 0)."""

    def __init__(self):
        self._last_sp: bytes | None = None

    def encode(self, buf: memoryview, seqs, is_prefill: bool, sp) -> int:
        from uno_b200.engine.noise import prompt_seed

        B = len(seqs)
        rows = np.empty((B, _FIELDS), dtype=np.int64)
        tables, tokens = [], []
        deterministic = getattr(sp, "noise_mode", None) == "deterministic_uniform"
        for i, s in enumerate(seqs):
            seed = prompt_seed(s) if deterministic else s.noise_seed
            mc = s.max_completion_tokens
            rows[i] = (s.seq_id, s.status.value, s.token_ids[-1], len(s.token_ids), s.num_prompt_tokens,
                       s.num_cached_tokens, -1 if mc is None else mc, seed is not None,
                       0 if seed is None else _i64(seed), len(s.block_table))
            tables.extend(s.block_table)
            if is_prefill:
                tokens.extend(s.token_ids)
        sp_bytes = pickle.dumps(sp, protocol=pickle.HIGHEST_PROTOCOL)
        send_sp = sp_bytes != self._last_sp
        self._last_sp = sp_bytes
        t = np.asarray(tables, dtype=np.int32)
        k = np.asarray(tokens, dtype=np.int32)
        head = np.array([MSG_RUN, int(is_prefill), B, len(sp_bytes) if send_sp else -1, t.size, k.size, 0, 0],
                        dtype=np.int64)
        off = 0
        for part in (head, rows, t, k):
            raw = part.tobytes()
            buf[off: off + len(raw)] = raw
            off += len(raw)
        if send_sp:
            buf[off: off + len(sp_bytes)] = sp_bytes
            off += len(sp_bytes)
        return off


class RunDecoder:
    """Rebuilds follower-side ``Sequence`` views from a packed ``run`` command."""

    def __init__(self):
        self._sp = None

    def decode(self, data: bytes):
        head = np.frombuffer(data, dtype=np.int64, count=8)
        _, is_prefill, B, sp_len, n_tab, n_tok = (int(x) for x in head[:6])
        off = 64
        rows = np.frombuffer(data, dtype=np.int64, count=B * _FIELDS, offset=off).reshape(B, _FIELDS)
        off += rows.nbytes
        tables = np.frombuffer(data, dtype=np.int32, count=n_tab, offset=off)
        off += tables.nbytes
        tokens = np.frombuffer(data, dtype=np.int32, count=n_tok, offset=off)
        off += tokens.nbytes
        if sp_len >= 0:
            self._sp = pickle.loads(data[off: off + sp_len])
        seqs = []
        tp = kp = 0
        for r in rows.tolist():
            seq_id, status, last, n, n_prompt, n_cached, mc, has_seed, seed, n_pages = r
            s = object.__new__(Sequence)
            s.seq_id = seq_id
            s.status = SequenceStatus(status)
            if is_prefill:
                s.token_ids = tokens[kp: kp + n].tolist()
                kp += n
            else:
                s.token_ids = TokenTail(n, last)
            s.num_prompt_tokens = n_prompt
            s.num_cached_tokens = n_cached
            s.block_table = tables[tp: tp + n_pages].tolist()
            tp += n_pages
            s.stats = new_decode_stats()
            s.max_completion_tokens = None if mc < 0 else mc
            s.noise_seed = (seed & 0xFFFFFFFFFFFFFFFF) if has_seed else None
            seqs.append(s)
        return seqs, bool(is_prefill), self._sp


class ChannelControlPlane:
    """``send(method, args)`` on rank 0, ``recv()`` on followers, over one ``CommandChannel``.

    ``group`` is the host (gloo) process group used for set-up and barriers.
    """

    def __init__(self, group, rank: int, world: int, channel: CommandChannel):
        self.group = group
        self.rank = rank
        self.world = world
        self.channel = channel
        self._enc = RunEncoder()
        self._dec = RunDecoder()

    @classmethod
    def create(cls, group, rank: int, world: int, timeout_s: float = 600.0):
        import torch.distributed as dist

        box = [None]
        if rank == 0:
            ch = CommandChannel(None, 0, world, size=channel_bytes(), timeout_s=timeout_s)
            box[0] = ch.name
        dist.broadcast_object_list(box, src=0, group=group)
        if rank != 0:
            ch = CommandChannel(box[0], rank, world, timeout_s=timeout_s)
        dist.barrier(group=group)  # every follower attached before rank 0 may unlink on failure
        return cls(group, rank, world, ch)

    def send(self, method: str, args: tuple) -> None:
        buf = self.channel.begin_write()
        if method == "run":
            seqs, is_prefill, sp = args
            n = self._enc.encode(buf, seqs, is_prefill, sp)
        else:
            raw = pickle.dumps((method, args), protocol=pickle.HIGHEST_PROTOCOL)
            head = np.array([MSG_PICKLE, len(raw), 0, 0, 0, 0, 0, 0], dtype=np.int64).tobytes()
            buf[: len(head)] = head
            buf[len(head): len(head) + len(raw)] = raw
            n = len(head) + len(raw)
        self.channel.commit(n)

    def recv(self):
        data = self.channel.read()
        kind = int(np.frombuffer(data, dtype=np.int64, count=1)[0])
        if kind == MSG_RUN:
            return "run", self._dec.decode(data)
        n = int(np.frombuffer(data, dtype=np.int64, count=2)[1])
        return pickle.loads(data[64: 64 + n])

    def close(self) -> None:
        self.channel.close()
