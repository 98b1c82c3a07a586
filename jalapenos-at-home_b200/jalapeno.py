"""Python binding of the B200 engine's C ABI (include/jalapeno.h).

The names mirror the reference engine crate's public Rust API
(engine/src/lib.rs:16-21): ``Model.load``, ``Model.cache``, ``Model.predict``,
``Model.hidden``, ``Model.next_token``, ``Model.generate``,
``DraftSchedule.fixed`` / ``DraftSchedule.adaptive``, ``generate_scheduled``,
``generate_speculative`` and ``SpeculativeResult``.  Every call goes through
``lib/libjalapeno.so``; there is no Python or CPU fallback, and importing this
module fails if the library has not been built.
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
# JALAPENO_LIB names another build of the library (the timeline build,
# lib/libjalapeno_timeline.so, for timeline.py)
LIB_PATH = Path(os.environ["JALAPENO_LIB"]) if os.environ.get("JALAPENO_LIB") else HERE / "lib" / "libjalapeno.so"

JL_OK, JL_ERR_INVALID_ARG, JL_ERR_FORMAT, JL_ERR_OOM = 0, 1, 2, 3
JL_ERR_CUDA, JL_ERR_TIMEOUT, JL_ERR_IO, JL_ERR_NO_DEVICE = 4, 5, 6, 7
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "FORMAT", 3: "OOM", 4: "CUDA", 5: "TIMEOUT",
                6: "IO", 7: "NO_DEVICE"}
KV_BF16, KV_F32 = 0, 1
SPEC_DEVICE, SPEC_HOST = 0, 1

# Symbols include/jalapeno.h declares (checked by tests).
EXPORTS = (
    "jl_last_error", "jl_version", "jl_device_count", "jl_weights_load", "jl_weights_free",
    "jl_weights_count", "jl_weights_at", "jl_weights_get", "jl_model_options_default",
    "jl_model_load", "jl_model_synthesize", "jl_model_free", "jl_model_info_get",
    "jl_model_read_tensor", "jl_cache_create", "jl_cache_free", "jl_cache_len",
    "jl_cache_truncate", "jl_predict", "jl_predict_draft", "jl_next_token", "jl_hidden", "jl_generate",
    "jl_schedule_fixed", "jl_schedule_adaptive", "jl_spec_options_default",
    "jl_generate_speculative", "jl_time_pass", "jl_time_projection", "jl_project",
    "jl_project_noalloc", "jl_pass_kernels", "jl_time_pass_draft", "jl_generate_batch",
    "jl_generate_speculative_batch", "jl_timeline_read", "jl_timeline_kernel", "jl_wait_probe",
    "jl_model_prompt_attention",
)
PROJ_QKV, PROJ_O, PROJ_GATE_UP, PROJ_DOWN, PROJ_HEAD = 0, 1, 2, 3, 4


class JlError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class TensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_size_t * 2), ("bf16", ctypes.POINTER(ctypes.c_uint16)),
                ("packed", ctypes.POINTER(ctypes.c_uint8)),
                ("scales", ctypes.POINTER(ctypes.c_uint8))]


class ModelOptions(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("kv_dtype", ctypes.c_int),
                ("kv_pool_tokens", ctypes.c_size_t), ("max_pass_rows", ctypes.c_size_t)]


class SynthConfig(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int), ("hidden", ctypes.c_int), ("q_heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("inter", ctypes.c_int), ("vocab", ctypes.c_int),
                ("tied", ctypes.c_int), ("max_positions", ctypes.c_int), ("eos", ctypes.c_int),
                ("seed", ctypes.c_uint64), ("mxfp4", ctypes.c_int), ("mxfp4_embed", ctypes.c_int)]


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("layers", "hidden", "q_heads", "kv_heads", "inter",
                                            "vocab", "max_positions", "eos", "tied",
                                            "mxfp4_projections", "mxfp4_head")] + \
               [("weight_bytes", ctypes.c_size_t), ("pass_bytes", ctypes.c_size_t),
                ("kv_bytes_per_token", ctypes.c_size_t)]


class Schedule(ctypes.Structure):
    _fields_ = [("gamma", ctypes.c_uint32), ("max_gamma", ctypes.c_uint32), ("adaptive", ctypes.c_int)]


class RoundStats(ctypes.Structure):
    _fields_ = [("gamma", ctypes.c_uint32), ("drafted", ctypes.c_uint32),
                ("accepted", ctypes.c_uint32), ("next_gamma", ctypes.c_uint32)]


class SpecOptions(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int), ("oracle_stream", ctypes.POINTER(ctypes.c_uint32)),
                ("oracle_len", ctypes.c_size_t), ("oracle_p", ctypes.c_double),
                ("oracle_seed", ctypes.c_uint64)]


class SpecResult(ctypes.Structure):
    _fields_ = [("tokens", ctypes.POINTER(ctypes.c_uint32)), ("tokens_cap", ctypes.c_size_t),
                ("rounds_out", ctypes.POINTER(RoundStats)), ("rounds_cap", ctypes.c_size_t),
                ("n_tokens", ctypes.c_size_t), ("drafted", ctypes.c_size_t),
                ("accepted", ctypes.c_size_t), ("rounds", ctypes.c_size_t),
                ("prefill_passes", ctypes.c_size_t), ("draft_passes", ctypes.c_size_t),
                ("verify_passes", ctypes.c_size_t), ("prefill_ms", ctypes.c_double),
                ("decode_ms", ctypes.c_double), ("draft_ms", ctypes.c_double),
                ("verify_ms", ctypes.c_double)]


class BatchStats(ctypes.Structure):
    _fields_ = [("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double), ("rounds", ctypes.c_size_t),
                ("target_passes", ctypes.c_size_t), ("draft_passes", ctypes.c_size_t)]


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` "
                          "(the engine has no CPU fallback)")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, sz, u32p = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint32)
    f32p = ctypes.POINTER(ctypes.c_float)
    sig = {
        "jl_last_error": ([], ctypes.c_char_p),
        "jl_version": ([], ctypes.c_char_p),
        "jl_device_count": ([], ctypes.c_int),
        "jl_weights_load": ([ctypes.c_char_p, ctypes.POINTER(vp)], ctypes.c_int),
        "jl_weights_free": ([vp], None),
        "jl_weights_count": ([vp], sz),
        "jl_weights_at": ([vp, sz, ctypes.POINTER(TensorView)], ctypes.c_int),
        "jl_weights_get": ([vp, ctypes.c_char_p, ctypes.POINTER(TensorView)], ctypes.c_int),
        "jl_model_options_default": ([ctypes.POINTER(ModelOptions)], None),
        "jl_model_load": ([ctypes.c_char_p, ctypes.POINTER(ModelOptions), ctypes.POINTER(vp)], ctypes.c_int),
        "jl_model_synthesize": ([ctypes.POINTER(SynthConfig), ctypes.POINTER(ModelOptions),
                                 ctypes.POINTER(vp)], ctypes.c_int),
        "jl_model_free": ([vp], None),
        "jl_model_info_get": ([vp, ctypes.POINTER(ModelInfo)], ctypes.c_int),
        "jl_model_read_tensor": ([vp, ctypes.c_char_p, vp, sz, ctypes.POINTER(sz)], ctypes.c_int),
        "jl_cache_create": ([vp, ctypes.POINTER(vp)], ctypes.c_int),
        "jl_cache_free": ([vp], None),
        "jl_cache_len": ([vp], sz),
        "jl_cache_truncate": ([vp, sz], ctypes.c_int),
        "jl_predict": ([vp, vp, u32p, sz, ctypes.c_int, u32p, f32p], ctypes.c_int),
        "jl_predict_draft": ([vp, vp, u32p, sz, u32p, f32p], ctypes.c_int),
        "jl_next_token": ([vp, u32p, sz, u32p], ctypes.c_int),
        "jl_hidden": ([vp, u32p, sz, sz, f32p], ctypes.c_int),
        "jl_generate": ([vp, u32p, sz, sz, u32p, sz, ctypes.POINTER(sz)], ctypes.c_int),
        "jl_schedule_fixed": ([ctypes.c_uint32, ctypes.POINTER(Schedule)], ctypes.c_int),
        "jl_schedule_adaptive": ([ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(Schedule)], ctypes.c_int),
        "jl_spec_options_default": ([ctypes.POINTER(SpecOptions)], None),
        "jl_generate_speculative": ([vp, vp, u32p, sz, sz, ctypes.POINTER(Schedule),
                                     ctypes.POINTER(SpecOptions), ctypes.POINTER(SpecResult)], ctypes.c_int),
        "jl_generate_batch": ([vp, sz, ctypes.POINTER(u32p), ctypes.POINTER(sz), sz, ctypes.POINTER(SpecResult),
                               ctypes.POINTER(BatchStats)], ctypes.c_int),
        "jl_generate_speculative_batch": ([vp, vp, sz, ctypes.POINTER(u32p), ctypes.POINTER(sz), sz,
                                           ctypes.POINTER(Schedule), ctypes.POINTER(SpecOptions),
                                           ctypes.POINTER(SpecResult), ctypes.POINTER(BatchStats)], ctypes.c_int),
        "jl_time_pass": ([vp, u32p, sz, sz, sz, ctypes.POINTER(ctypes.c_double),
                          ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
        "jl_time_projection": ([vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                ctypes.POINTER(ctypes.c_double), ctypes.POINTER(sz)], ctypes.c_int),
        "jl_project": ([vp, ctypes.c_int, ctypes.c_int, f32p, sz, f32p], ctypes.c_int),
        "jl_project_noalloc": ([vp, ctypes.c_int, ctypes.c_int, vp, sz, vp, vp], ctypes.c_int),
        "jl_pass_kernels": ([vp, sz, ctypes.c_int, ctypes.POINTER(sz)], ctypes.c_int),
        "jl_time_pass_draft": ([vp, u32p, sz, sz, ctypes.POINTER(ctypes.c_double),
                                ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
        "jl_timeline_read": ([ctypes.POINTER(ctypes.c_uint64), sz, ctypes.POINTER(sz)], ctypes.c_int),
        "jl_timeline_kernel": ([sz], ctypes.c_char_p),
        "jl_wait_probe": ([vp, ctypes.c_uint32], ctypes.c_int),
        "jl_model_prompt_attention": ([vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    return L


lib = _load()


def check(status: int) -> None:
    if status != JL_OK:
        raise JlError(status, lib.jl_last_error().decode(errors="replace"))


def u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64).astype(np.uint32))


def _p(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def device_count() -> int:
    return lib.jl_device_count()


# ---------------------------------------------------------------------------
# host weights: engine::load (engine/src/lib.rs:85-202)


class Weights:
    """``Weights``: tensors read from a checkpoint directory on the host."""

    def __init__(self, directory: str | os.PathLike):
        h = ctypes.c_void_p()
        check(lib.jl_weights_load(str(directory).encode(), ctypes.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            lib.jl_weights_free(self._h)
            self._h = None

    def __len__(self) -> int:
        return lib.jl_weights_count(self._h)

    def names(self) -> list[str]:
        out = []
        for i in range(len(self)):
            v = TensorView()
            check(lib.jl_weights_at(self._h, i, ctypes.byref(v)))
            out.append(v.name.decode())
        return out

    def tensor(self, name: str) -> dict:
        v = TensorView()
        check(lib.jl_weights_get(self._h, name.encode(), ctypes.byref(v)))
        shape = tuple(v.shape[i] for i in range(v.ndim))
        n = int(np.prod(shape))
        if v.dtype == 1:
            return {"dtype": "mxfp4", "shape": shape,
                    "packed": np.ctypeslib.as_array(v.packed, (n // 2,)).copy(),
                    "scales": np.ctypeslib.as_array(v.scales, (n // 32,)).copy()}
        return {"dtype": "bf16", "shape": shape, "bf16": np.ctypeslib.as_array(v.bf16, (n,)).copy()}


def load(directory) -> Weights:
    """``engine::load`` (lib.rs:85-87)."""
    return Weights(directory)


# ---------------------------------------------------------------------------
# models: Model (engine/src/model.rs)


def model_options(kv_dtype: int = KV_BF16, kv_pool_tokens: int = 0, max_pass_rows: int = 0,
                  device: int = 0) -> ModelOptions:
    o = ModelOptions()
    lib.jl_model_options_default(ctypes.byref(o))
    o.device = device
    o.kv_dtype = kv_dtype
    o.kv_pool_tokens = kv_pool_tokens
    o.max_pass_rows = max_pass_rows
    return o


class Model:
    """A model resident on one GPU (``Model`` with ``Backend::Gpu``)."""

    def __init__(self, handle: ctypes.c_void_p, name: str):
        self._h = handle
        self.name = name
        info = ModelInfo()
        check(lib.jl_model_info_get(self._h, ctypes.byref(info)))
        self.info = info

    @classmethod
    def load(cls, directory, **opts) -> "Model":
        """``Model::load`` (model.rs:55-57)."""
        h = ctypes.c_void_p()
        o = model_options(**opts)
        check(lib.jl_model_load(str(directory).encode(), ctypes.byref(o), ctypes.byref(h)))
        return cls(h, str(directory))

    @classmethod
    def synthesize(cls, layers, hidden, q_heads, kv_heads, inter, vocab, tied, seed, mxfp4=False,
                   mxfp4_embed=False, max_positions=40960, eos=151645, name=None, **opts) -> "Model":
        c = SynthConfig(layers, hidden, q_heads, kv_heads, inter, vocab, int(tied), max_positions,
                        eos, seed, int(mxfp4), int(mxfp4_embed))
        h = ctypes.c_void_p()
        o = model_options(**opts)
        check(lib.jl_model_synthesize(ctypes.byref(c), ctypes.byref(o), ctypes.byref(h)))
        return cls(h, name or f"synthetic-seed{seed}")

    @classmethod
    def from_config(cls, cfg, seed: int, mxfp4: bool = False, **opts) -> "Model":
        """Seeded synthetic weights for an architecture with fields layers,
        hidden, q_heads, kv_heads, inter, vocab, tied, max_positions, eos."""
        return cls.synthesize(cfg.layers, cfg.hidden, cfg.q_heads, cfg.kv_heads, cfg.inter,
                              cfg.vocab, cfg.tied, seed, mxfp4=mxfp4,
                              max_positions=cfg.max_positions, eos=cfg.eos,
                              name=f"{cfg.name}{'-MXFP4' if mxfp4 else ''}/seed{seed}", **opts)

    def __del__(self):
        if getattr(self, "_h", None):
            lib.jl_model_free(self._h)
            self._h = None

    def free(self) -> None:
        self.__del__()

    @property
    def eos(self) -> int:
        return self.info.eos

    @property
    def vocab(self) -> int:
        return self.info.vocab

    def context_limit(self) -> int:
        return self.info.max_positions

    def cache(self) -> "Cache":
        """``Model::cache`` (model.rs:124-133)."""
        return Cache(self)

    def predict(self, tokens, cache: "Cache", all: bool = False, logits: bool = False):
        """``Model::predict`` (model.rs:209-240)."""
        t = u32(tokens)
        rows = len(t) if all else 1
        ids = np.zeros(rows, np.uint32)
        lg = np.empty((rows, self.vocab), np.float32) if logits else None
        check(lib.jl_predict(self._h, cache._h, _p(t, ctypes.c_uint32), len(t), int(all),
                             _p(ids, ctypes.c_uint32), None if lg is None else _p(lg, ctypes.c_float)))
        out = [int(i) for i in ids]
        return (out, lg) if logits else out

    def predict_draft(self, tokens, cache: "Cache", logits: bool = False):
        """One draft step (1 or 2 tokens, predicting after the last) through
        the kernels a speculative loop's draft passes run: the proposal
        passes of ``generate_scheduled`` (speculative.rs:84-92, 136-138)."""
        t = u32(tokens)
        out = np.zeros(1, np.uint32)
        lg = np.empty((1, self.vocab), np.float32) if logits else None
        check(lib.jl_predict_draft(self._h, cache._h, _p(t, ctypes.c_uint32), len(t),
                                   _p(out, ctypes.c_uint32),
                                   None if lg is None else _p(lg, ctypes.c_float)))
        return ([int(out[0])], lg) if logits else [int(out[0])]

    @property
    def has_draft_path(self) -> bool:
        """Whether draft steps take kernels of their own (CUDA-core MXFP4
        projections) rather than the tensor-core pass every other pass takes."""
        return self.pass_kernels(1, draft_step=True) != self.pass_kernels(1)

    def next_token(self, tokens) -> int:
        """``Model::next_token`` (model.rs:203-205)."""
        t = u32(tokens)
        out = ctypes.c_uint32()
        check(lib.jl_next_token(self._h, _p(t, ctypes.c_uint32), len(t), ctypes.byref(out)))
        return int(out.value)

    def hidden(self, tokens, layers: int) -> np.ndarray:
        """``Model::hidden`` (model.rs:143-154)."""
        t = u32(tokens)
        out = np.empty((len(t), self.info.hidden), np.float32)
        check(lib.jl_hidden(self._h, _p(t, ctypes.c_uint32), len(t), layers, _p(out, ctypes.c_float)))
        return out

    def generate(self, prompt, count: int) -> list[int]:
        """``Model::generate`` (model.rs:268-285)."""
        t = u32(prompt)
        cap = len(t) + count
        out = np.zeros(max(cap, 1), np.uint32)
        n = ctypes.c_size_t()
        check(lib.jl_generate(self._h, _p(t, ctypes.c_uint32), len(t), count,
                              _p(out, ctypes.c_uint32), cap, ctypes.byref(n)))
        return [int(x) for x in out[: n.value]]

    def time_pass(self, prompt, rows: int, reps: int = 15) -> tuple[float, float]:
        """``Model::time_pass`` (model.rs:242-266): median (wall_ms, gpu_ms)."""
        t = u32(prompt)
        wall, gpu = ctypes.c_double(), ctypes.c_double()
        check(lib.jl_time_pass(self._h, _p(t, ctypes.c_uint32), len(t), rows, reps,
                               ctypes.byref(wall), ctypes.byref(gpu)))
        return wall.value, gpu.value

    def project(self, layer: int, which: int, x) -> np.ndarray:
        """One layer projection as the pass runs it (``matmul``, lib.rs:240-266,
        in its fused forms); see jl_project in include/jalapeno.h."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        widths = {PROJ_QKV: (self.info.q_heads + 2 * self.info.kv_heads) * 128,
                  PROJ_O: self.info.hidden, PROJ_GATE_UP: self.info.inter,
                  PROJ_DOWN: self.info.hidden, PROJ_HEAD: self.info.vocab}
        y = np.empty((x.shape[0], widths[which]), np.float32)
        check(lib.jl_project(self._h, layer, which, _p(x, ctypes.c_float), x.shape[0],
                             _p(y, ctypes.c_float)))
        return y

    def project_noalloc(self, layer: int, which: int, x_ptr: int, rows: int, y_ptr: int,
                        stream: int = 0) -> None:
        """jl_project on device memory the caller owns, with no allocation:
        ``x_ptr``/``y_ptr`` are device addresses of f32 [rows, width] arrays
        (widths as for :meth:`project`), ``stream`` a cudaStream_t handle or 0
        for the model's stream.  See jl_project_noalloc in include/jalapeno.h."""
        check(lib.jl_project_noalloc(self._h, layer, which, ctypes.c_void_p(x_ptr), rows,
                                     ctypes.c_void_p(y_ptr), ctypes.c_void_p(stream or None)))

    def time_pass_draft(self, prompt, reps: int = 15) -> tuple[float, float]:
        """time_pass of one row on the draft-step path: median (wall_ms, gpu_ms)."""
        t = u32(prompt)
        wall, gpu = ctypes.c_double(), ctypes.c_double()
        check(lib.jl_time_pass_draft(self._h, _p(t, ctypes.c_uint32), len(t), reps,
                                     ctypes.byref(wall), ctypes.byref(gpu)))
        return wall.value, gpu.value

    def prompt_attention(self, tensor_cores: bool = True) -> bool:
        """Kernel of the prompt attention for later prompt passes: tcgen05
        MMAs (default, where the model allows) or CUDA cores.  Returns whether
        prompts now run on tensor cores."""
        active = ctypes.c_int(0)
        check(lib.jl_model_prompt_attention(self._h, int(bool(tensor_cores)), ctypes.byref(active)))
        return bool(active.value)

    def wait_probe(self, polls: int = 1000) -> None:
        """One device wait that nothing completes, bounded by ``polls`` polls:
        raises JlError(JL_ERR_TIMEOUT) and leaves the model usable."""
        check(lib.jl_wait_probe(self._h, polls))

    def pass_kernels(self, rows: int, draft_step: bool = False) -> int:
        """Kernels one forward pass of `rows` rows launches (see jl_pass_kernels)."""
        n = ctypes.c_size_t()
        check(lib.jl_pass_kernels(self._h, rows, int(draft_step), ctypes.byref(n)))
        return n.value

    def time_projection(self, layer: int, which: int, rows: int, iters: int = 20) -> tuple[float, int]:
        """Mean device ms per launch of one projection kernel, and its weight bytes."""
        ms, nb = ctypes.c_double(), ctypes.c_size_t()
        check(lib.jl_time_projection(self._h, layer, which, rows, iters, ctypes.byref(ms),
                                     ctypes.byref(nb)))
        return ms.value, nb.value

    def read_tensor(self, name: str, nbytes: int) -> np.ndarray:
        buf = np.empty(nbytes, np.uint8)
        n = ctypes.c_size_t()
        check(lib.jl_model_read_tensor(self._h, name.encode(), buf.ctypes.data_as(ctypes.c_void_p),
                                       nbytes, ctypes.byref(n)))
        return buf[: n.value]


class Cache:
    """``KvCache`` (model.rs:37-52) on the GPU."""

    def __init__(self, model: Model):
        self._model = model
        h = ctypes.c_void_p()
        check(lib.jl_cache_create(model._h, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            lib.jl_cache_free(self._h)
            self._h = None

    @property
    def len(self) -> int:
        return lib.jl_cache_len(self._h)

    def truncate(self, n: int) -> None:
        check(lib.jl_cache_truncate(self._h, n))


# ---------------------------------------------------------------------------
# speculative decoding (engine/src/speculative.rs, engine/src/scheduler.rs)


class DraftSchedule:
    """``DraftSchedule`` (scheduler.rs:1-27)."""

    def __init__(self, s: Schedule):
        self._s = s

    @classmethod
    def fixed(cls, gamma: int) -> "DraftSchedule":
        s = Schedule()
        check(lib.jl_schedule_fixed(gamma, ctypes.byref(s)))
        return cls(s)

    @classmethod
    def adaptive(cls, initial: int, maximum: int) -> "DraftSchedule":
        s = Schedule()
        check(lib.jl_schedule_adaptive(initial, maximum, ctypes.byref(s)))
        return cls(s)

    @property
    def gamma(self) -> int:
        return self._s.gamma


@dataclasses.dataclass
class PhaseStats:
    passes: int
    elapsed_ms: float


@dataclasses.dataclass
class SpeculativeResult:
    """``SpeculativeResult`` (speculative.rs:21-30)."""
    tokens: list
    drafted: int
    accepted: int
    rounds: int
    prefill: PhaseStats
    draft: PhaseStats
    verify: PhaseStats
    round_stats: list
    decode_ms: float


def generate_scheduled(target: Model, draft: Model, prompt, count: int, schedule: DraftSchedule,
                       mode: int = SPEC_DEVICE, oracle_stream=None, oracle_p: float = 0.0,
                       oracle_seed: int = 0) -> SpeculativeResult:
    """``generate_scheduled`` (speculative.rs:43-143)."""
    t = u32(prompt)
    cap = len(t) + count + 1
    toks = np.zeros(cap, np.uint32)
    rounds = (RoundStats * (count + 2))()
    res = SpecResult()
    res.tokens = _p(toks, ctypes.c_uint32)
    res.tokens_cap = cap
    res.rounds_out = rounds
    res.rounds_cap = count + 2
    o = SpecOptions()
    lib.jl_spec_options_default(ctypes.byref(o))
    o.mode = mode
    stream = None
    if oracle_stream is not None:
        stream = u32(oracle_stream)
        o.oracle_stream = _p(stream, ctypes.c_uint32)
        o.oracle_len = len(stream)
        o.oracle_p = oracle_p
        o.oracle_seed = oracle_seed
    check(lib.jl_generate_speculative(target._h, draft._h, _p(t, ctypes.c_uint32), len(t), count,
                                      ctypes.byref(schedule._s), ctypes.byref(o), ctypes.byref(res)))
    n = min(res.rounds, res.rounds_cap)
    return SpeculativeResult(
        tokens=[int(x) for x in toks[: res.n_tokens]], drafted=res.drafted, accepted=res.accepted,
        rounds=res.rounds, prefill=PhaseStats(res.prefill_passes, res.prefill_ms),
        draft=PhaseStats(res.draft_passes, res.draft_ms),
        verify=PhaseStats(res.verify_passes, res.verify_ms),
        round_stats=[(r.gamma, r.drafted, r.accepted, r.next_gamma) for r in rounds[:n]],
        decode_ms=res.decode_ms)


def generate_speculative(target: Model, draft: Model, prompt, count: int, gamma: int,
                         **kw) -> SpeculativeResult:
    """``generate_speculative`` (speculative.rs:32-40)."""
    return generate_scheduled(target, draft, prompt, count, DraftSchedule.fixed(gamma), **kw)


@dataclasses.dataclass
class BatchResult:
    """A batched call: one result per sequence, and the batch's own counters."""
    results: list        # SpeculativeResult per sequence (greedy: tokens and verify passes)
    prefill_ms: float
    decode_ms: float
    rounds: int
    target_passes: int   # passes of up to 16 rows
    draft_passes: int


def _batch_inputs(prompts, count, rounds_cap=0):
    ps = [u32(p) for p in prompts]
    ptrs = (ctypes.POINTER(ctypes.c_uint32) * len(ps))(*[_p(p, ctypes.c_uint32) for p in ps])
    lens = (ctypes.c_size_t * len(ps))(*[len(p) for p in ps])
    outs = [np.zeros(len(p) + count + 1, np.uint32) for p in ps]
    rounds = [(RoundStats * rounds_cap)() for _ in ps] if rounds_cap else []
    res = (SpecResult * len(ps))()
    for i, o in enumerate(outs):
        res[i].tokens = _p(o, ctypes.c_uint32)
        res[i].tokens_cap = len(o)
        if rounds_cap:
            res[i].rounds_out = rounds[i]
            res[i].rounds_cap = rounds_cap
    return ps, ptrs, lens, outs, rounds, res


def _batch_result(outs, rounds, res, stats) -> BatchResult:
    seqs = []
    for i, o in enumerate(outs):
        r = res[i]
        n = min(r.rounds, r.rounds_cap)
        seqs.append(SpeculativeResult(
            tokens=[int(x) for x in o[: r.n_tokens]], drafted=r.drafted, accepted=r.accepted, rounds=r.rounds,
            prefill=PhaseStats(r.prefill_passes, r.prefill_ms), draft=PhaseStats(r.draft_passes, r.draft_ms),
            verify=PhaseStats(r.verify_passes, r.verify_ms),
            round_stats=[(x.gamma, x.drafted, x.accepted, x.next_gamma) for x in rounds[i][:n]] if rounds else [],
            decode_ms=r.decode_ms))
    return BatchResult(seqs, stats.prefill_ms, stats.decode_ms, stats.rounds, stats.target_passes,
                       stats.draft_passes)


def generate_batch(model: Model, prompts, count: int) -> BatchResult:
    """Greedy ``generate`` (model.rs:268-285) of independent sequences in
    lockstep rounds: each sequence's tokens equal ``model.generate`` on it."""
    ps, ptrs, lens, outs, rounds, res = _batch_inputs(prompts, count)
    stats = BatchStats()
    check(lib.jl_generate_batch(model._h, len(ps), ptrs, lens, count, res, ctypes.byref(stats)))
    return _batch_result(outs, rounds, res, stats)


def generate_speculative_batch(target: Model, draft: Model, prompts, count: int, schedule,
                               oracle_streams=None, oracle_p=0.0, oracle_seeds=0) -> BatchResult:
    """``generate_scheduled`` (speculative.rs:43-143) for each of a batch of
    sequences in lockstep rounds.  ``schedule``, ``oracle_p`` and
    ``oracle_seeds`` may be one value for all sequences or one per sequence;
    ``oracle_streams`` is None or one stream (or None) per sequence."""
    B = len(prompts)
    per = lambda v: list(v) if isinstance(v, (list, tuple)) else [v] * B
    scheds = per(schedule)
    ps, ptrs, lens, outs, rounds, res = _batch_inputs(prompts, count, rounds_cap=count + 2)
    sc = (Schedule * B)(*[(s._s if isinstance(s, DraftSchedule) else DraftSchedule.fixed(s)._s) for s in scheds])
    opts = (SpecOptions * B)()
    keep = []
    streams = oracle_streams if oracle_streams is not None else [None] * B
    for i, (st, p, seed) in enumerate(zip(streams, per(oracle_p), per(oracle_seeds))):
        lib.jl_spec_options_default(ctypes.byref(opts[i]))
        if st is not None:
            a = u32(st)
            keep.append(a)
            opts[i].oracle_stream = _p(a, ctypes.c_uint32)
            opts[i].oracle_len = len(a)
            opts[i].oracle_p = p
            opts[i].oracle_seed = seed
    stats = BatchStats()
    check(lib.jl_generate_speculative_batch(target._h, draft._h, B, ptrs, lens, count, sc, opts, res,
                                            ctypes.byref(stats)))
    return _batch_result(outs, rounds, res, stats)


def _philox4x32_10(c0, c1, c2, c3, k0: int, k1: int):
    """Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1,
    2, 3", SC 2011) over arrays of counters, in uint64 lanes."""
    m = np.uint64(0xFFFFFFFF)
    c = [np.asarray(x, np.uint64) & m for x in (c0, c1, c2, c3)]
    k0, k1 = np.uint64(k0), np.uint64(k1)
    for r in range(10):
        if r:
            k0 = (k0 + np.uint64(0x9E3779B9)) & m
            k1 = (k1 + np.uint64(0xBB67AE85)) & m
        p0 = np.uint64(0xD2511F53) * c[0]
        p1 = np.uint64(0xCD9E8D57) * c[2]
        c = [(p1 >> np.uint64(32)) ^ c[1] ^ k0, p1 & m, (p0 >> np.uint64(32)) ^ c[3] ^ k1, p0 & m]
    return c


def prompt_ids(n: int, vocab: int, seed: int) -> list[int]:
    """Seeded uniform prompt ids for synthetic workloads: id 4i+j is word j
    of Philox4x32-10 at counter (i, 0, 0, "prmp") under key (seed, "toks"),
    modulo the vocabulary."""
    i = np.arange((n + 3) // 4, dtype=np.uint64)
    z = np.zeros_like(i)
    w = _philox4x32_10(i, z, z, z + np.uint64(0x70726D70), seed & 0xFFFFFFFF, 0x746F6B73)
    ids = np.stack(w, axis=1).reshape(-1)[:n] % np.uint64(vocab)
    return [int(x) for x in ids]


TIMELINE_CTAS, TIMELINE_POINTS = 512, 8


def timeline() -> tuple[list[str], np.ndarray]:
    """Kernel names and stamps [launch][cta][point] (GPU nanoseconds, 0 where
    nothing stamped) of the last recorded pass: jl_timeline_read, from the
    timeline build of the library only (JALAPENO_LIB)."""
    n = ctypes.c_size_t()
    check(lib.jl_timeline_read(None, 0, ctypes.byref(n)))
    buf = np.zeros((n.value, TIMELINE_CTAS, TIMELINE_POINTS), dtype=np.uint64)
    check(lib.jl_timeline_read(_p(buf, ctypes.c_uint64), buf.size, ctypes.byref(n)))
    names = [lib.jl_timeline_kernel(i).decode() for i in range(n.value)]
    return names, buf

