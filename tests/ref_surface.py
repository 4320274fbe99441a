"""A communicator that exposes nothing beyond collab_infer's ``Communicator`` surface
(``distributed/comm.py:200-630``): what ``CollabEngine``'s own ``ParallelContext`` hands to the
attention call sites.  Wraps one of this package's communicators, so it runs on any backend."""

REFERENCE_SURFACE = frozenset({
    "ranks", "size", "global_rank", "rank", "group", "name", "device", "backend", "comm_device", "stats",
    "emulator", "small_message_bytes", "comm_dtype", "activation_dtype", "is_trivial", "to_wire", "wire_dtype",
    "all_reduce", "all_gather_list", "all_gather", "reduce_scatter", "all_to_all", "broadcast", "broadcast_object",
    "barrier", "isend", "irecv", "send", "recv",
})


class ReferenceSurfaceComm:
    def __init__(self, inner):
        self.__dict__["_inner"] = inner

    def __getattr__(self, name):
        if name in REFERENCE_SURFACE:
            return getattr(self.__dict__["_inner"], name)
        raise AttributeError(f"collab_infer's Communicator has no attribute {name!r}")
