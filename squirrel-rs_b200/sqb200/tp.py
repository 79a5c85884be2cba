"""Host-side plumbing of a tensor-parallel group (one process per GPU).

Before any NCCL or GPU work the ranks check in through the process group's
key-value store, so a rank that died or never started is found on the host and
named, instead of every other rank blocking inside ncclCommInitRank (which waits
for all ranks without a time limit). Rank 0 then publishes the NCCL unique id
through the same store. Between phases, `check_in` with a new tag tells the ranks
whether a peer left, before anyone launches the next collective.

Keys are never reused: every Group gets a generation number (the count of groups
this process made on the same key prefix, which is the same on every rank because
every rank runs the same program), and every use of a check-in tag or of share_id
inside a group is numbered too. A second group, a repeated tag or a second
share_id therefore waits for fresh keys instead of passing at once on keys an
earlier phase left in the store (which could hand a rank a stale NCCL id).

    grp = Group.from_default_store(timeout_s=120)   # after dist.init_process_group
    nccl_id = grp.share_id(lib.nccl_unique_id)
    model = lib.Model(path, device=local, tp_rank=grp.rank, tp_size=grp.world, nccl_id=nccl_id)
"""
import datetime


class GroupTimeout(TimeoutError):
    """A rank of the group did not arrive in time (the ranks that are missing, if known)."""

    def __init__(self, msg, missing=None):
        super().__init__(msg)
        self.missing = list(missing or [])


class Group:
    _generations = {}  # key prefix -> groups made so far in this process

    def __init__(self, store, rank: int, world: int, timeout_s: float = 120.0, prefix: str = "sqb200/tp",
                 generation: int = None):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = float(timeout_s)
        if generation is None:
            generation = Group._generations.get(prefix, 0)
            Group._generations[prefix] = generation + 1
        self.prefix = f"{prefix}/g{generation}"
        self._uses = {}

    @classmethod
    def from_default_store(cls, timeout_s: float = 120.0):
        """The group of the default torch.distributed process group, on its store."""
        import torch.distributed as dist
        from torch.distributed import distributed_c10d as c10d
        return cls(c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), timeout_s)

    def _key(self, *parts):
        return "/".join([self.prefix] + [str(p) for p in parts])

    def _use(self, name):
        """A fresh name for the n-th use of `name` in this group."""
        n = self._uses.get(name, 0)
        self._uses[name] = n + 1
        return f"{name}#{n}"

    def _wait(self, keys, what):
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception as e:  # the store raises on expiry; name who is missing
            missing = [k for k in keys if not self.store.check([k])]
            raise GroupTimeout(f"tensor-parallel group: {what} not there within {self.timeout_s:g} s "
                               f"(rank {self.rank} of {self.world}; missing {missing})",
                               missing) from e

    def check_in(self, tag: str):
        """Every rank announces itself under `tag` and waits for all the others.
        Raises GroupTimeout naming the ranks that did not arrive."""
        name = self._use(tag)
        self.store.set(self._key(name, self.rank), b"1")
        keys = [self._key(name, r) for r in range(self.world)]
        try:
            self._wait(keys, f"check-in '{tag}'")
        except GroupTimeout as e:
            ranks = [int(k.rsplit("/", 1)[1]) for k in e.missing]
            raise GroupTimeout(f"tensor-parallel group: rank(s) {ranks} did not check in at '{tag}' within "
                               f"{self.timeout_s:g} s (seen from rank {self.rank} of {self.world})", ranks) from e

    def share_id(self, make_id) -> bytes:
        """Check in, then rank 0 makes the NCCL unique id (make_id()) and every rank
        returns the same bytes."""
        self.check_in("init")
        key = self._key(self._use("nccl_id"))
        if self.rank == 0:
            self.store.set(key, bytes(make_id()))
        self._wait([key], "the NCCL id from rank 0")
        return bytes(self.store.get(key))
