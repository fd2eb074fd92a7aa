"""Python bindings of the armcc SDK C API (include/armcc_sdk.h) exported by
libsg_b200.so: load a package, select its "cuda" graph, run sessions."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

ARMCC_OK = 0


class ArmDeviceState(ctypes.Structure):
    _fields_ = [("soc_id", ctypes.c_int), ("ram_mb", ctypes.c_uint32), ("battery_pct", ctypes.c_int32),
                ("thermal_state", ctypes.c_int), ("latency_mode", ctypes.c_int),
                ("context_length", ctypes.c_uint32), ("gpu_available", ctypes.c_bool),
                ("npu_available", ctypes.c_bool)]


class ArmSessionOptions(ctypes.Structure):
    _fields_ = [("num_threads", ctypes.c_int32), ("use_gpu", ctypes.c_bool), ("use_npu", ctypes.c_bool),
                ("seed", ctypes.c_uint32), ("verbose", ctypes.c_bool)]


class ArmInferenceResult(ctypes.Structure):
    _fields_ = [("next_token_id", ctypes.c_int32), ("logprob", ctypes.c_float), ("ttft_ms", ctypes.c_float),
                ("tpot_ms", ctypes.c_float), ("tokens_generated", ctypes.c_uint32), ("status", ctypes.c_int)]


class ArmPackageInfo(ctypes.Structure):
    _fields_ = [("model_id", ctypes.c_char * 256), ("model_family", ctypes.c_char * 64),
                ("compiler_version", ctypes.c_char * 32), ("num_graphs", ctypes.c_uint32),
                ("num_kernels", ctypes.c_uint32), ("num_weight_files", ctypes.c_uint32),
                ("num_layers", ctypes.c_uint32), ("hidden_size", ctypes.c_uint32),
                ("vocab_size", ctypes.c_uint32)]


class SgTpModel(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab", "group_size")]


class SgTpShard(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("q_head0", "q_head1", "kv_head0", "kv_head1", "ffn0", "ffn1",
                                              "vocab0", "vocab1")]


_P = ctypes.c_void_p
_CB = ctypes.CFUNCTYPE(None, ctypes.c_int32, ctypes.c_void_p)
_SIGS = {
    "armpack_load": (_P, [ctypes.c_char_p]),
    "armpack_destroy": (None, [_P]),
    "armpack_last_error": (ctypes.c_char_p, []),
    "armpack_select_graph": (_P, [_P, ctypes.POINTER(ArmDeviceState)]),
    "armpack_num_graphs": (ctypes.c_uint32, [_P]),
    "armpack_get_graph": (_P, [_P, ctypes.c_uint32]),
    "armgraph_description": (ctypes.c_char_p, [_P]),
    "armgraph_estimated_tpot_ms": (ctypes.c_float, [_P]),
    "armgraph_peak_memory_bytes": (ctypes.c_uint64, [_P]),
    "armgraph_create_session": (_P, [_P, ctypes.POINTER(ArmSessionOptions)]),
    "armsess_destroy": (None, [_P]),
    "armsess_reset": (None, [_P]),
    "armsess_prefill": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32]),
    "armsess_decode": (ArmInferenceResult, [_P]),
    "armsess_generate": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32, ctypes.c_uint32,
                                        _CB, _P]),
    "armgraph_run": (ArmInferenceResult, [_P, ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32]),
    "armpack_get_info": (ctypes.c_int, [_P, ctypes.POINTER(ArmPackageInfo)]),
    "armpack_print_summary": (None, [_P]),
    "armpack_get_tokenizer": (_P, [_P]),
    "sg_session_last_logits": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_float), ctypes.c_uint32]),
    "sg_session_position": (ctypes.c_uint32, [_P]),
    "sg_select_graph_within": (_P, [_P, ctypes.POINTER(ArmDeviceState), ctypes.c_uint64]),
    "sg_graph_session_bytes": (ctypes.c_uint64, [_P, ctypes.c_uint32]),
    "sg_tp_shard": (ctypes.c_int, [ctypes.POINTER(SgTpModel), ctypes.c_int32, ctypes.c_int32,
                                   ctypes.POINTER(SgTpShard)]),
    "sg_tp_unique_id": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint8)]),
    "sg_session_create_tp": (_P, [_P, ctypes.POINTER(ArmSessionOptions), ctypes.c_int32, ctypes.c_int32,
                                  ctypes.POINTER(ctypes.c_uint8)]),
    "sg_session_vocab_range": (None, [_P, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)]),
    "sg_session_create_paged": (_P, [_P, ctypes.POINTER(ArmSessionOptions), ctypes.c_uint32, ctypes.c_uint64,
                                     ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint8)]),
    "sg_session_abort": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "sg_session_kv_pages": (ctypes.c_int32, [_P, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)]),
    "sg_session_step_kernel": (ctypes.c_int32, [_P, ctypes.POINTER(ctypes.c_char_p)]),
    "sg_session_step_trace": (ctypes.c_int32, [_P, ctypes.c_int32, _P, ctypes.c_uint32,
                                               ctypes.POINTER(ctypes.c_int32)]),
    "sg_session_step_gpu_ms": (ctypes.c_double, [_P, ctypes.c_int32]),
    "sg_session_graph_kernels": (ctypes.c_int32, [_P]),
    "sg_session_create_ex": (_P, [_P, ctypes.POINTER(ArmSessionOptions), ctypes.c_uint32, ctypes.c_int32,
                                  ctypes.c_int32, ctypes.POINTER(ctypes.c_uint8)]),
    "sg_batch_prefill": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32]),
    "sg_batch_decode": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "sg_session_batch": (ctypes.c_uint32, [_P]),
}


class ArmError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"armcc status {status}: {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    L = _lib.load()
    if not getattr(L, "_armcc_sigs", False):
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        L._armcc_sigs = True
    return L


def last_error() -> str:
    return (lib().armpack_last_error() or b"").decode(errors="replace")


def _tokens(tokens) -> tuple[ctypes.Array, int]:
    a = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), a.size, a


def tp_shard(cfg: dict, rank: int, world: int, group_size: int) -> dict:
    """The tensor-parallel shard of `rank` among `world` for a model config
    (silicongraph_b200.armpack.llama_config keys); host only."""
    m = SgTpModel(cfg["hidden_size"], cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"],
                  cfg["intermediate_size"], cfg["vocab_size"], group_size)
    out = SgTpShard()
    st = lib().sg_tp_shard(ctypes.byref(m), rank, world, ctypes.byref(out))
    if st != ARMCC_OK:
        raise ArmError(st, last_error())
    return {f: getattr(out, f) for f, _ in SgTpShard._fields_}


def tp_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for sessions of one tensor-parallel group."""
    buf = (ctypes.c_uint8 * 128)()
    st = lib().sg_tp_unique_id(buf)
    if st != ARMCC_OK:
        raise ArmError(st, last_error())
    return bytes(buf)


class Package:
    def __init__(self, path: str):
        self.h = lib().armpack_load(path.encode())
        if not self.h:
            raise ArmError(-2, last_error())

    def close(self):
        if self.h:
            lib().armpack_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def num_graphs(self) -> int:
        return lib().armpack_num_graphs(self.h)

    def info(self) -> dict:
        i = ArmPackageInfo()
        st = lib().armpack_get_info(self.h, ctypes.byref(i))
        if st != ARMCC_OK:
            raise ArmError(st, last_error())
        return {f: (getattr(i, f).decode() if isinstance(getattr(i, f), bytes) else getattr(i, f))
                for f, _ in ArmPackageInfo._fields_}

    def graph(self, index: int) -> "Graph":
        g = lib().armpack_get_graph(self.h, index)
        if not g:
            raise ArmError(-1, last_error())
        return Graph(self, g)

    def select(self, context_length: int = 0, *, ram_mb: int = 0, thermal: int = 0, latency: int = 0,
               device_bytes_available: int | None = None) -> "Graph":
        """armpack_select_graph: the best-scoring graph whose session fits in
        95 % of the device memory available (free memory now, capped by
        ram_mb when given); with device_bytes_available, against that figure
        instead (sg_select_graph_within, no device query)."""
        st = ArmDeviceState(gpu_available=True, context_length=context_length, ram_mb=ram_mb,
                            thermal_state=thermal, latency_mode=latency)
        if device_bytes_available is None:
            g = lib().armpack_select_graph(self.h, ctypes.byref(st))
        else:
            g = lib().sg_select_graph_within(self.h, ctypes.byref(st), device_bytes_available)
        if not g:
            raise ArmError(-1, last_error())
        return Graph(self, g)


class Graph:
    def __init__(self, pkg: Package, h):
        self.pkg, self.h = pkg, h

    @property
    def description(self) -> str:
        return lib().armgraph_description(self.h).decode()

    @property
    def peak_memory_bytes(self) -> int:
        return lib().armgraph_peak_memory_bytes(self.h)

    def session_bytes(self, batch: int = 1) -> int:
        """Device bytes a session of `batch` sequences allocates (one slab)."""
        return lib().sg_graph_session_bytes(self.h, batch)

    def session(self, tp: tuple[int, int, bytes] | None = None, batch: int = 1,
                kv_pool_tokens: int | None = None) -> "Session":
        """A session; tp = (rank, world, unique id) joins a tensor-parallel group;
        batch > 1 decodes that many sequences in lockstep; kv_pool_tokens pages
        the KV cache with a pool of that many tokens over all sequences (0:
        every sequence's full context)."""
        return Session(self, tp, batch, kv_pool_tokens)

    def run(self, tokens) -> ArmInferenceResult:
        p, n, _keep = _tokens(tokens)
        return lib().armgraph_run(self.h, p, n)


class Session:
    def __init__(self, graph: Graph, tp: tuple[int, int, bytes] | None = None, batch: int = 1,
                 kv_pool_tokens: int | None = None):
        self.graph = graph
        if kv_pool_tokens is not None:
            rank, world, uid = tp if tp is not None else (0, 1, bytes(128))
            buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
            self.h = lib().sg_session_create_paged(graph.h, None, batch, kv_pool_tokens, rank, world, buf)
        elif tp is None and batch == 1:
            self.h = lib().armgraph_create_session(graph.h, None)
        else:
            rank, world, uid = tp if tp is not None else (0, 1, bytes(128))
            buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
            self.h = lib().sg_session_create_ex(graph.h, None, batch, rank, world, buf)
        if not self.h:
            raise ArmError(-5, last_error())

    def close(self):
        if self.h:
            lib().armsess_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        lib().armsess_reset(self.h)

    def prefill(self, tokens):
        p, n, _keep = _tokens(tokens)
        st = lib().armsess_prefill(self.h, p, n)
        if st != ARMCC_OK:
            raise ArmError(st, last_error())

    def decode(self) -> ArmInferenceResult:
        r = lib().armsess_decode(self.h)
        if r.status != ARMCC_OK:
            raise ArmError(r.status, last_error())
        return r

    def generate(self, prompt, max_new_tokens: int) -> list[int]:
        out = []
        cb = _CB(lambda tok, ctx: out.append(int(tok)))
        p, n, _keep = _tokens(prompt)
        st = lib().armsess_generate(self.h, p, n, max_new_tokens, cb, None)
        if st != ARMCC_OK:
            raise ArmError(st, last_error())
        return out

    @property
    def batch(self) -> int:
        return lib().sg_session_batch(self.h)

    def batch_prefill(self, tokens) -> None:
        """tokens [batch, n]: one prompt per sequence, all of length n."""
        a = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        if a.ndim != 2 or a.shape[0] != self.batch:
            raise ValueError(f"tokens must be [{self.batch}, n]")
        st = lib().sg_batch_prefill(self.h, a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), a.shape[1])
        if st != ARMCC_OK:
            raise ArmError(st, last_error())

    def batch_decode(self) -> np.ndarray:
        """Every sequence's next greedy token."""
        out = np.zeros(self.batch, np.int32)
        st = lib().sg_batch_decode(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
        if st != ARMCC_OK:
            raise ArmError(st, last_error())
        return out

    def last_logits(self, vocab: int | None = None) -> np.ndarray:
        """fp32 logits of the last processed token over vocab_range (the first
        `vocab` of them when given)."""
        if vocab is None:
            lo, hi = self.vocab_range
            vocab = (hi - lo) * self.batch
        out = np.zeros(vocab, np.float32)
        st = lib().sg_session_last_logits(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), vocab)
        if st != ARMCC_OK:
            raise ArmError(st, last_error())
        return out

    def abort(self, reason: str = "") -> None:
        """sg_session_abort: end the session's tensor-parallel group; later calls are refused."""
        st = lib().sg_session_abort(self.h, reason.encode())
        if st != ARMCC_OK:
            raise ArmError(st, last_error())

    @property
    def kv_pages(self) -> tuple[int, int] | None:
        """(pages in the pool, pages in use) of a paged KV cache, None when flat."""
        pool, used = ctypes.c_uint32(), ctypes.c_uint32()
        if not lib().sg_session_kv_pages(self.h, ctypes.byref(pool), ctypes.byref(used)):
            return None
        return pool.value, used.value

    @property
    def step_kernel(self) -> tuple[bool, str | None]:
        """(whether one-token steps run as the persistent decode-step kernel, why not)."""
        why = ctypes.c_char_p()
        on = bool(lib().sg_session_step_kernel(self.h, ctypes.byref(why)))
        return on, (why.value.decode() if why.value else None)

    @property
    def graph_kernels(self) -> int:
        """Kernel launches in one captured decode step (-1 before capture or when eager)."""
        return lib().sg_session_graph_kernels(self.h)

    def step_gpu_ms(self, on: bool) -> float:
        """Device time of decode steps: step_gpu_ms(True) starts timing;
        step_gpu_ms(False) stops and returns the mean ms per step."""
        v = lib().sg_session_step_gpu_ms(self.h, 1 if on else 0)
        if v < 0:
            raise ArmError(-5, last_error())
        return v

    def step_trace(self, on: bool = True):
        """Decode-step kernel timeline: step_trace(True) records the following
        steps; step_trace(False) returns the last step's stamps as an int64
        array [cta][512] (ns) and stops."""
        import numpy as np
        n_ct = ctypes.c_int32()
        if on:
            if lib().sg_session_step_trace(self.h, 1, None, 0, ctypes.byref(n_ct)) < 0:
                raise ArmError(-5, last_error())
            return None
        lib().sg_session_step_trace(self.h, 1, None, 0, ctypes.byref(n_ct))
        out = np.zeros(n_ct.value * 512, np.uint64)
        n = lib().sg_session_step_trace(self.h, 1, out.ctypes.data, out.size, ctypes.byref(n_ct))
        lib().sg_session_step_trace(self.h, 0, None, 0, ctypes.byref(n_ct))
        if n < 0:
            raise ArmError(-5, last_error())
        return out.reshape(n_ct.value, 512).astype(np.int64)

    @property
    def position(self) -> int:
        return lib().sg_session_position(self.h)

    @property
    def vocab_range(self) -> tuple[int, int]:
        """[lo, hi) of the logits last_logits returns (a shard on a tensor-parallel session)."""
        lo, hi = ctypes.c_uint32(), ctypes.c_uint32()
        lib().sg_session_vocab_range(self.h, ctypes.byref(lo), ctypes.byref(hi))
        return lo.value, hi.value
