"""penumbra_b200 -- Python host binding of the B200 encrypted-evaluation library.

Every call goes through the C ABI of ``libpenumbra_b200.so`` (``include/penumbra_b200.h``);
PyTorch only supplies device memory and the current CUDA stream.  There is no CPU fallback:
importing this package without the built library raises.

The names mirror the reference runtime's public surface (``runtime/src/lib.rs:36-45``):
``keygen`` (``keys.rs:47``), ``encrypt`` / ``decrypt_vec`` (``encrypt.rs:20-45``), and the
per-op kernels that replace tfhe-rs calls inside ``Linear``/``Conv2d``/``Requant``/``Activation``.
"""
from __future__ import annotations

import ctypes as C
import math
import os

import torch

__all__ = [
    "Params", "default_params", "params_n8192", "KeySet", "keygen", "lib", "LibraryError",
    "encrypt", "phase", "decrypt_vec", "test_vector", "keyswitch", "keyswitch_workspace_bytes",
    "pbs_batch", "blind_rotate",
    "pbs_workspace_bytes", "lwe_contract", "lwe_contract_gather", "fft_negacyclic_mul", "measure_fp64_peak",
    "device_status", "pbs_batch_noalloc", "Graph", "Plan", "Evaluator", "shard",
    "gather_shards", "evaluate_sharded", "op_bits", "wait_probe", "import_keys", "radix_merge",
    "TensorDesc", "KeyRing", "op_plan", "requant_batch", "argmax_batch", "add_batch",
    "radix_plan", "lwe_contract_ld", "lwe_contract_gather_ld", "deserialize_keys",
    "serialize_lwe", "deserialize_lwe",
]

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpenumbra_b200.so")


class LibraryError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


class Params(C.Structure):
    """``pnb_params`` (field meaning of tfhe-rs ClassicPBSParameters)."""
    _fields_ = [
        ("n", C.c_int32), ("k", C.c_int32), ("N", C.c_int32),
        ("pbs_base_log", C.c_int32), ("pbs_level", C.c_int32),
        ("ks_base_log", C.c_int32), ("ks_level", C.c_int32),
        ("msg_bits", C.c_int32), ("carry_bits", C.c_int32), ("reserved", C.c_int32),
        ("lwe_std", C.c_double), ("glwe_std", C.c_double),
    ]

    def delta(self) -> int:
        """Plaintext scaling: one padding bit above msg_bits + carry_bits."""
        return 1 << (63 - self.msg_bits - self.carry_bits)

    def as_tuple(self):
        return tuple(getattr(self, f) for f, _ in self._fields_)


_SIGS = {
    "pnb_version": (C.c_int, []),
    "pnb_last_error": (C.c_char_p, []),
    "pnb_params_default": (C.c_int, [C.POINTER(Params)]),
    "pnb_params_n8192": (C.c_int, [C.POINTER(Params)]),
    "pnb_keygen": (C.c_int, [C.c_int, C.POINTER(Params), C.c_uint64, C.POINTER(C.c_void_p)]),
    "pnb_keys_free": (C.c_int, [C.c_void_p]),
    "pnb_keys_import": (C.c_int, [C.c_int, C.POINTER(Params), C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "pnb_keys_info": (C.c_int, [C.c_void_p, C.POINTER(Params), C.POINTER(C.c_int),
                                C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "pnb_keys_export": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "pnb_encrypt_lwe": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64,
                                  C.c_void_p, C.c_int, C.c_void_p]),
    "pnb_phase_lwe": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                C.c_void_p]),
    "pnb_test_vector": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_uint64, C.c_void_p,
                                  C.c_void_p]),
    "pnb_keyswitch_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int]),
    "pnb_keyswitch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                C.c_size_t, C.c_void_p]),
    "pnb_blind_rotate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_void_p]),
    "pnb_pbs_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int]),
    "pnb_pbs_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                C.c_void_p, C.c_size_t, C.c_void_p]),
    "pnb_pbs_batch_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_void_p]),
    "pnb_radix_merge": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                  C.c_void_p, C.c_void_p]),
    "pnb_lwe_contract_gather": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int,
                                          C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                          C.c_void_p]),
    "pnb_lwe_contract": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int,
                                   C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "pnb_lwe_contract_ld": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int,
                                      C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                      C.c_void_p]),
    "pnb_lwe_contract_gather_ld": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int,
                                             C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                             C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "pnb_keys_serialized_bytes": (C.c_size_t, [C.c_void_p, C.c_int]),
    "pnb_keys_serialize": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t]),
    "pnb_keys_deserialize": (C.c_int, [C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    "pnb_lwe_serialized_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "pnb_lwe_serialize": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "pnb_lwe_deserialize": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                      C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "pnb_fft_negacyclic_mul": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_int, C.c_void_p]),
    "pnb_measure_fp64_peak": (C.c_int, [C.c_int, C.POINTER(C.c_double)]),
    "pnb_device_status": (C.c_int, [C.c_int, C.POINTER(C.c_int)]),
    "pnb_wait_probe": (C.c_int, [C.c_int, C.c_uint, C.POINTER(C.c_int)]),
    "pnb_graph_load": (C.c_int, [C.c_char_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    "pnb_graph_free": (C.c_int, [C.c_void_p]),
    "pnb_graph_info": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                 C.POINTER(C.c_int)]),
    "pnb_graph_check_budget": (C.c_int, [C.c_void_p]),
    "pnb_op_bits": (C.c_int, [C.c_char_p, C.c_size_t, C.POINTER(C.c_int), C.c_int,
                             C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "pnb_plan_create": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                  C.c_double, C.POINTER(C.c_void_p)]),
    "pnb_plan_free": (C.c_int, [C.c_void_p]),
    "pnb_plan_info": (C.c_int, [C.c_void_p, C.c_void_p]),
    "pnb_plan_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int64),
                                  C.POINTER(C.c_int), C.POINTER(C.c_int64),
                                  C.POINTER(C.c_int64)]),
    "pnb_plan_report": (C.c_size_t, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "pnb_plan_key_sets": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                    C.POINTER(C.c_int64)]),
    "pnb_plan_simulate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                    C.POINTER(C.c_double)]),
    "pnb_evaluator_create": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64, C.c_size_t,
                                       C.POINTER(C.c_void_p)]),
    "pnb_evaluator_free": (C.c_int, [C.c_void_p]),
    "pnb_evaluator_keys": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "pnb_evaluator_reserve": (C.c_int, [C.c_void_p, C.c_int]),
    "pnb_evaluate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "pnb_keyring_create": (C.c_int, [C.c_int, C.POINTER(Params), C.c_uint64,
                                     C.POINTER(C.c_void_p)]),
    "pnb_keyring_free": (C.c_int, [C.c_void_p]),
    "pnb_keyring_keys": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]),
    "pnb_op_plan_create": (C.c_int, [C.c_char_p, C.c_size_t, C.POINTER(Params), C.c_void_p,
                                     C.c_int, C.c_int, C.c_double, C.c_double,
                                     C.POINTER(C.c_void_p)]),
    "pnb_plan_tensor_desc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "pnb_radix_plan_create": (C.c_int, [C.POINTER(Params), C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_void_p, C.c_double, C.POINTER(C.c_void_p)]),
    "pnb_evaluator_create_with": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.POINTER(C.c_void_p)]),
    "pnb_requant_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                    C.c_int, C.c_double, C.c_void_p, C.c_void_p, C.c_void_p]),
    "pnb_argmax_batch": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_int, C.c_double, C.c_void_p, C.c_void_p, C.c_void_p]),
    "pnb_add_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_int, C.c_int, C.c_double, C.c_void_p, C.c_void_p,
                                C.c_void_p]),
    "pnb_shard": (C.c_int, [C.c_int64, C.c_int, C.c_int, C.POINTER(C.c_int64),
                            C.POINTER(C.c_int64)]),
    "pnb_comm_unique_id": (C.c_int, [C.c_void_p]),
    "pnb_comm_create": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p,
                                  C.POINTER(C.c_void_p)]),
    "pnb_comm_free": (C.c_int, [C.c_void_p]),
    "pnb_comm_abort": (C.c_int, [C.c_void_p]),
    "pnb_comm_info": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                C.POINTER(C.c_int)]),
    "pnb_comm_status": (C.c_int, [C.c_void_p]),
    "pnb_allgather": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                C.c_void_p]),
}

_LIB = None


def lib() -> C.CDLL:
    """Load ``libpenumbra_b200.so``; raise if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C {_HERE}` (or "
                "__graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


def _check(fn: str, rc: int):
    if rc != 0:
        msg = lib().pnb_last_error().decode(errors="replace")
        raise LibraryError(fn, rc, msg)


def _stream(device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    if t is None:
        return C.c_void_p(0)
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return C.c_void_p(t.data_ptr())


def default_params() -> Params:
    p = Params()
    _check("pnb_params_default", lib().pnb_params_default(C.byref(p)))
    return p


def params_n8192() -> Params:
    """The library's 6-bit set at N = 8192 (``pnb_params_n8192``)."""
    p = Params()
    _check("pnb_params_n8192", lib().pnb_params_n8192(C.byref(p)))
    return p


class KeySet:
    """Keys resident on one GPU (``pnb_keys``): Fourier BSK, KSK and client secrets."""

    def __init__(self, handle: C.c_void_p, params: Params, device: int, seed: int,
                 owner=None):
        self._h = handle
        self.params = params
        self.device = device
        self.seed = seed
        self._owner = owner  # a borrowed key set keeps its owner alive and never frees

    @property
    def handle(self) -> C.c_void_p:
        if not self._h:
            raise ValueError("key set has been freed")
        return self._h

    def free(self):
        if self._h and self._owner is None:
            lib().pnb_keys_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:  # interpreter shutdown
            pass

    @property
    def big_dim(self) -> int:
        return self.params.k * self.params.N

    def info(self) -> dict:
        p = Params()
        dev = C.c_int()
        fb = C.c_size_t()
        kb = C.c_size_t()
        _check("pnb_keys_info",
               lib().pnb_keys_info(self.handle, C.byref(p), C.byref(dev), C.byref(fb),
                                   C.byref(kb)))
        return {"device": dev.value, "fourier_bsk_bytes": fb.value, "ksk_bytes": kb.value}

    def serialize(self, with_secrets: bool = False) -> bytes:
        """The key set as a byte container (``pnb_keys_serialize``); without secrets it carries
        the evaluation keys only."""
        n = lib().pnb_keys_serialized_bytes(self.handle, int(with_secrets))
        buf = C.create_string_buffer(n)
        _check("pnb_keys_serialize", lib().pnb_keys_serialize(self.handle, int(with_secrets),
                                                              buf, n))
        return buf.raw

    def export(self, lwe_sk=True, glwe_sk=True, bsk=False, ksk=False) -> dict:
        """Copy key material to host numpy arrays (blocking)."""
        import numpy as np
        p = self.params
        rows = (p.k + 1) * p.pbs_level
        out = {}
        bufs = []
        for name, want, size in (
                ("lwe_sk", lwe_sk, p.n), ("glwe_sk", glwe_sk, p.k * p.N),
                ("bsk", bsk, p.n * rows * (p.k + 1) * p.N),
                ("ksk", ksk, p.k * p.N * p.ks_level * (p.n + 1))):
            if want:
                a = np.zeros(size, dtype=np.uint64)
                out[name] = a
                bufs.append(C.c_void_p(a.ctypes.data))
            else:
                bufs.append(C.c_void_p(0))
        _check("pnb_keys_export", lib().pnb_keys_export(self.handle, *bufs))
        return out


def keygen(params: Params | None = None, seed: int = 0, device: int = 0) -> KeySet:
    """Generate keys on ``device`` (blocking).  Mirrors ``keys::keygen`` (keys.rs:47)."""
    params = default_params() if params is None else params
    h = C.c_void_p()
    _check("pnb_keygen", lib().pnb_keygen(device, C.byref(params), seed, C.byref(h)))
    return KeySet(h, params, device, seed)


def import_keys(params: Params, keys: dict, device: int = 0) -> KeySet:
    """Key set from host arrays in ``KeySet.export`` layouts (``bsk`` and ``ksk`` required;
    ``lwe_sk`` and ``glwe_sk`` optional, together).  Mirrors ``pnb_keys_import``."""
    import numpy as np
    bufs = []
    for name in ("lwe_sk", "glwe_sk", "bsk", "ksk"):
        a = keys.get(name)
        if a is None:
            bufs.append(C.c_void_p(0))
        else:
            a = np.ascontiguousarray(a, dtype=np.uint64)
            keys = dict(keys, **{name: a})  # keep the converted array alive during the call
            bufs.append(C.c_void_p(a.ctypes.data))
    h = C.c_void_p()
    _check("pnb_keys_import",
           lib().pnb_keys_import(device, C.byref(params), *bufs, C.byref(h)))
    return KeySet(h, params, device, 0)


def deserialize_keys(data: bytes, device: int = 0) -> KeySet:
    """A key set from ``KeySet.serialize`` bytes (``pnb_keys_deserialize``)."""
    h = C.c_void_p()
    _check("pnb_keys_deserialize", lib().pnb_keys_deserialize(device, data, len(data),
                                                              C.byref(h)))
    p, dev = Params(), C.c_int()
    fb, kb = C.c_size_t(), C.c_size_t()
    _check("pnb_keys_info", lib().pnb_keys_info(h, C.byref(p), C.byref(dev), C.byref(fb),
                                                C.byref(kb)))
    return KeySet(h, p, device, 0)


def serialize_lwe(ct) -> bytes:
    """LWE ciphertexts [count, dim+1] (torch tensor or numpy array) as a byte container."""
    import numpy as np
    a = ct.cpu().numpy() if isinstance(ct, torch.Tensor) else np.asarray(ct)
    a = np.ascontiguousarray(a.reshape(-1, a.shape[-1])).view(np.uint64)
    count, dim = a.shape[0], a.shape[1] - 1
    n = lib().pnb_lwe_serialized_bytes(count, dim)
    buf = C.create_string_buffer(n)
    _check("pnb_lwe_serialize", lib().pnb_lwe_serialize(C.c_void_p(a.ctypes.data), count, dim,
                                                        buf, n))
    return buf.raw


def deserialize_lwe(data: bytes):
    """Ciphertexts [count, dim+1] (numpy u64) from ``serialize_lwe`` bytes."""
    import numpy as np
    count, dim = C.c_int(), C.c_int()
    _check("pnb_lwe_deserialize", lib().pnb_lwe_deserialize(data, len(data), None, 0,
                                                            C.byref(count), C.byref(dim)))
    out = np.zeros((count.value, dim.value + 1), dtype=np.uint64)
    _check("pnb_lwe_deserialize", lib().pnb_lwe_deserialize(data, len(data),
                                                            C.c_void_p(out.ctypes.data),
                                                            out.size, C.byref(count),
                                                            C.byref(dim)))
    return out


def _u64(t: torch.Tensor) -> torch.Tensor:
    """View an int64 tensor as the u64 words the C ABI expects (torch has no uint64 math)."""
    if t.dtype not in (torch.int64, torch.uint64):
        raise TypeError(f"expected a 64-bit tensor, got {t.dtype}")
    return t


def encrypt(keys: KeySet, messages: torch.Tensor, seed: int, first_index: int = 0,
            delta: int | None = None) -> torch.Tensor:
    """LWE-encrypt ``messages * delta`` under the big key; returns [count, k*N+1] int64."""
    dev = torch.device("cuda", keys.device)
    msg = messages.to(device=dev, dtype=torch.int64).contiguous()
    count = msg.numel()
    ct = torch.empty((count, keys.big_dim + 1), dtype=torch.int64, device=dev)
    delta = keys.params.delta() if delta is None else delta
    _check("pnb_encrypt_lwe",
           lib().pnb_encrypt_lwe(keys.handle, _ptr(msg), delta % (1 << 64), seed, first_index,
                                 _ptr(ct), count, _stream(dev)))
    return ct


def phase(keys: KeySet, ct: torch.Tensor, small_key: bool = False) -> torch.Tensor:
    """Phase ``b - <a, s>`` of each ciphertext (int64 view of the u64 torus value)."""
    ct = _u64(ct).contiguous()
    dim = keys.params.n if small_key else keys.big_dim
    count = ct.numel() // (dim + 1)
    out = torch.empty(count, dtype=torch.int64, device=ct.device)
    _check("pnb_phase_lwe",
           lib().pnb_phase_lwe(keys.handle, _ptr(ct), _ptr(out), count, int(small_key),
                               _stream(ct.device)))
    return out


def decode(params: Params, phases: torch.Tensor, delta: int | None = None,
           space: int | None = None) -> torch.Tensor:
    """Round phases to the nearest multiple of ``delta`` and reduce modulo ``space``."""
    delta = params.delta() if delta is None else delta
    space = (2 << (params.msg_bits + params.carry_bits)) if space is None else space
    shift = delta.bit_length() - 1
    assert delta == 1 << shift, "delta must be a power of two"
    ph = phases.to(torch.int64)
    # round(phase / delta) with wrapping u64 arithmetic expressed in int64
    r = torch.bitwise_right_shift(ph + (1 << (shift - 1)), shift)
    return torch.remainder(r, space)


def decrypt_vec(keys: KeySet, ct: torch.Tensor, delta: int | None = None,
                space: int | None = None) -> torch.Tensor:
    """Decrypt to integers.  Mirrors ``encrypt::decrypt_vec`` (encrypt.rs:43-45)."""
    return decode(keys.params, phase(keys, ct), delta, space)


def test_vector(keys: KeySet, lut, delta_out: int | None = None) -> torch.Tensor:
    """Blind-rotation test vector of ``lut`` (``generate_lookup_table``)."""
    import numpy as np
    dev = torch.device("cuda", keys.device)
    lut_a = np.ascontiguousarray(np.asarray(lut, dtype=np.int64).astype(np.uint64))
    tv = torch.empty(keys.params.N, dtype=torch.int64, device=dev)
    delta_out = keys.params.delta() if delta_out is None else delta_out
    _check("pnb_test_vector",
           lib().pnb_test_vector(keys.handle, C.c_void_p(lut_a.ctypes.data), len(lut_a),
                                 delta_out % (1 << 64), _ptr(tv), _stream(dev)))
    return tv


def keyswitch_workspace_bytes(keys: KeySet, count: int) -> int:
    return int(lib().pnb_keyswitch_workspace_bytes(keys.handle, count))


def keyswitch(keys: KeySet, ct: torch.Tensor, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Keyswitch big-key ciphertexts [count, k*N+1] to the small key [count, n+1]."""
    ct = _u64(ct).contiguous()
    count = ct.numel() // (keys.big_dim + 1)
    if out is None:
        out = torch.empty((count, keys.params.n + 1), dtype=torch.int64, device=ct.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check("pnb_keyswitch",
           lib().pnb_keyswitch(keys.handle, _ptr(ct), _ptr(out), count, _ptr(workspace),
                               ws_bytes, _stream(ct.device)))
    return out


def blind_rotate(keys: KeySet, tv: torch.Tensor, small: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Blind rotation + sample extraction of small-key ciphertexts [count, n+1]."""
    small = _u64(small).contiguous()
    count = small.numel() // (keys.params.n + 1)
    if out is None:
        out = torch.empty((count, keys.big_dim + 1), dtype=torch.int64, device=small.device)
    _check("pnb_blind_rotate",
           lib().pnb_blind_rotate(keys.handle, _ptr(tv), _ptr(small), _ptr(out), count,
                                  _stream(small.device)))
    return out


def pbs_workspace_bytes(keys: KeySet, count: int) -> int:
    return int(lib().pnb_pbs_workspace_bytes(keys.handle, count))


def pbs_batch(keys: KeySet, tv: torch.Tensor, ct: torch.Tensor,
              out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Programmable bootstrap of every ciphertext (``apply_lookup_table`` batched)."""
    ct = _u64(ct).contiguous()
    count = ct.numel() // (keys.big_dim + 1)
    if out is None:
        out = torch.empty((count, keys.big_dim + 1), dtype=torch.int64, device=ct.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check("pnb_pbs_batch",
           lib().pnb_pbs_batch(keys.handle, _ptr(tv), _ptr(ct), _ptr(out), count,
                               _ptr(workspace), ws_bytes, _stream(ct.device)))
    return out


def pbs_batch_noalloc(keys: KeySet, tv: torch.Tensor, ct: torch.Tensor,
                      out: torch.Tensor) -> torch.Tensor:
    """Bootstrap into a caller-provided ``out`` with no device allocation inside the library.

    For callers that cannot allocate GPU memory on this path; the library's fixed 4 MiB
    scratch limits a call to 247 ciphertexts with the default parameters, and concurrent calls
    on the GPU race on that scratch.
    """
    ct = _u64(ct).contiguous()
    count = ct.numel() // (keys.big_dim + 1)
    _check("pnb_pbs_batch_noalloc",
           lib().pnb_pbs_batch_noalloc(keys.handle, _ptr(tv), _ptr(ct), _ptr(out), count,
                                       _stream(ct.device)))
    return out


def radix_merge(keys: KeySet, blocks: torch.Tensor, delta_out: int, signed: bool = True,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge radix integers ``blocks[count, num_blocks, kN+1]`` (block 0 least significant, one
    digit per block at the reference's block delta) into wide ciphertexts ``[count, kN+1]``
    encrypting each integer times ``delta_out``: one bootstrap per block, then a sum."""
    blocks = _u64(blocks).contiguous()
    count, nb, L = blocks.shape
    if L != keys.big_dim + 1:
        raise ValueError(f"blocks have {L} words, the key set's ciphertexts {keys.big_dim + 1}")
    if out is None:
        out = torch.empty((count, L), dtype=torch.int64, device=blocks.device)
    _check("pnb_radix_merge",
           lib().pnb_radix_merge(keys.handle, _ptr(blocks), nb, count, int(bool(signed)),
                                 delta_out % (1 << 64), _ptr(out), _stream(blocks.device)))
    return out


def lwe_contract(W: torch.Tensor, bias: torch.Tensor | None, delta: int, X: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """``Y[b, j, :] = sum_i W[j, i] X[b, i, :] + bias[j] * delta`` on the body (mod 2^64)."""
    if W.dtype != torch.int8:
        raise TypeError("W must be int8")
    M, K = W.shape
    B, K2, L = X.shape
    if K2 != K:
        raise ValueError(f"X has {K2} inputs, W expects {K}")
    if out is None:
        out = torch.empty((B, M, L), dtype=torch.int64, device=X.device)
    bias_t = None if bias is None else bias.to(device=X.device, dtype=torch.int64).contiguous()
    with torch.cuda.device(X.device):
        _check("pnb_lwe_contract",
               lib().pnb_lwe_contract(_ptr(W.contiguous()), _ptr(bias_t), delta % (1 << 64), M,
                                      K, _ptr(_u64(X).contiguous()), _ptr(out), B, L,
                                      _stream(X.device)))
    return out


def lwe_contract_gather(W: torch.Tensor, bias: torch.Tensor | None, delta: int,
                        X: torch.Tensor, index: torch.Tensor,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """``Y[g, j, :] = sum_k W[j, k] X[index[g, k], :] + bias[j] * delta`` (index -1 = zero)."""
    if W.dtype != torch.int8 or index.dtype != torch.int32:
        raise TypeError("W must be int8 and index int32")
    M, K = W.shape
    G, K2 = index.shape
    if K2 != K:
        raise ValueError(f"index has {K2} taps, W expects {K}")
    L = X.shape[-1]
    if out is None:
        out = torch.empty((G, M, L), dtype=torch.int64, device=X.device)
    bias_t = None if bias is None else bias.to(device=X.device, dtype=torch.int64).contiguous()
    with torch.cuda.device(X.device):
        _check("pnb_lwe_contract_gather",
               lib().pnb_lwe_contract_gather(_ptr(W.contiguous()), _ptr(bias_t),
                                             delta % (1 << 64), M, K,
                                             _ptr(_u64(X).contiguous()),
                                             _ptr(index.contiguous()), G, _ptr(out), L,
                                             _stream(X.device)))
    return out


def lwe_contract_ld(W: torch.Tensor, bias: torch.Tensor | None, delta: int, X: torch.Tensor,
                    lwe_len: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """``lwe_contract`` over rows at a pitch: X [B, K, ldx] holds ``lwe_len`` words per row
    (ldx >= lwe_len); the result is [B, M, ldx] at the same pitch (words past ``lwe_len`` are
    left as they were)."""
    if W.dtype != torch.int8:
        raise TypeError("W must be int8")
    M, K = W.shape
    B, K2, ld = X.shape
    if K2 != K:
        raise ValueError(f"X has {K2} inputs, W expects {K}")
    if out is None:
        out = torch.zeros((B, M, ld), dtype=torch.int64, device=X.device)
    bias_t = None if bias is None else bias.to(device=X.device, dtype=torch.int64).contiguous()
    with torch.cuda.device(X.device):
        _check("pnb_lwe_contract_ld",
               lib().pnb_lwe_contract_ld(_ptr(W.contiguous()), _ptr(bias_t), delta % (1 << 64),
                                         M, K, _ptr(_u64(X).contiguous()), ld, _ptr(out),
                                         out.shape[-1], B, lwe_len, _stream(X.device)))
    return out


def lwe_contract_gather_ld(W: torch.Tensor, bias: torch.Tensor | None, delta: int,
                           X: torch.Tensor, index: torch.Tensor, lwe_len: int,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """``lwe_contract_gather`` over rows at a pitch (X [*, ldx]; result [G, M, ldx])."""
    if W.dtype != torch.int8 or index.dtype != torch.int32:
        raise TypeError("W must be int8 and index int32")
    M, K = W.shape
    G, K2 = index.shape
    if K2 != K:
        raise ValueError(f"index has {K2} taps, W expects {K}")
    ld = X.shape[-1]
    if out is None:
        out = torch.zeros((G, M, ld), dtype=torch.int64, device=X.device)
    bias_t = None if bias is None else bias.to(device=X.device, dtype=torch.int64).contiguous()
    with torch.cuda.device(X.device):
        _check("pnb_lwe_contract_gather_ld",
               lib().pnb_lwe_contract_gather_ld(_ptr(W.contiguous()), _ptr(bias_t),
                                                delta % (1 << 64), M, K,
                                                _ptr(_u64(X).contiguous()), ld,
                                                _ptr(index.contiguous()), G, _ptr(out),
                                                out.shape[-1], lwe_len, _stream(X.device)))
    return out


def fft_negacyclic_mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Negacyclic products through the blind rotation's f64 FFT (diagnostic)."""
    count, N = a.shape
    out = torch.empty_like(b)
    _check("pnb_fft_negacyclic_mul",
           lib().pnb_fft_negacyclic_mul(a.device.index or 0, N, _ptr(a.contiguous()),
                                        _ptr(b.contiguous()), _ptr(out), count,
                                        _stream(a.device)))
    return out


def device_status(device: int = 0) -> int:
    """Read and clear the tensor-core kernels' status word (0 = every bounded wait completed)."""
    v = C.c_int()
    _check("pnb_device_status", lib().pnb_device_status(device, C.byref(v)))
    return v.value


def op_bits(op: dict, input_bits: list[int]) -> tuple[int, int]:
    """(output bits, internal bits) of one IR op consuming tensors of the given widths."""
    import json as _json
    text = _json.dumps(op).encode()
    arr = (C.c_int * max(len(input_bits), 1))(*input_bits)
    out, internal = C.c_int(), C.c_int()
    _check("pnb_op_bits", lib().pnb_op_bits(text, len(text), arr, len(input_bits),
                                            C.byref(out), C.byref(internal)))
    return out.value, internal.value


def wait_probe(device: int = 0, polls: int = 1000) -> int:
    """Warps of a probe kernel that gave up a bounded wait on a never-completed barrier."""
    v = C.c_int()
    _check("pnb_wait_probe", lib().pnb_wait_probe(device, polls, C.byref(v)))
    return v.value


def measure_fp64_peak(device: int = 0) -> float:
    v = C.c_double()
    _check("pnb_measure_fp64_peak", lib().pnb_measure_fp64_peak(device, C.byref(v)))
    return v.value


# ---- graph evaluation ------------------------------------------------------------------------

class _PlanSummary(C.Structure):
    _fields_ = [("input_elems", C.c_int64), ("output_elems", C.c_int64),
                ("num_inputs", C.c_int32), ("num_outputs", C.c_int32),
                ("pbs_per_sample", C.c_int64), ("cost_per_sample", C.c_double),
                ("num_instructions", C.c_int32), ("reserved", C.c_int32)]


class Graph:
    """An IR graph (``model.fhe``), parsed and validated by the library.

    Mirrors ``Graph::from_json`` + ``OpSpec::build`` (runtime/src/ir.rs:169-180, 197-452);
    errors raise ``LibraryError`` carrying the reference's diagnosis."""

    def __init__(self, doc):
        import json as _json
        if isinstance(doc, dict):
            doc = _json.dumps(doc)
        if isinstance(doc, str):
            doc = doc.encode()
        h = C.c_void_p()
        _check("pnb_graph_load", lib().pnb_graph_load(doc, len(doc), C.byref(h)))
        self._h = h

    def check_budget(self):
        """``check_graph_bit_width_budget`` (runtime/src/eval.rs:237-276)."""
        _check("pnb_graph_check_budget", lib().pnb_graph_check_budget(self._h))

    def info(self) -> dict:
        a, b, c = C.c_int(), C.c_int(), C.c_int()
        _check("pnb_graph_info", lib().pnb_graph_info(self._h, C.byref(a), C.byref(b), C.byref(c)))
        return {"num_nodes": a.value, "num_blocks": b.value, "input_bits": c.value}

    def __del__(self):
        try:
            if self._h:
                lib().pnb_graph_free(self._h)
                self._h = None
        except Exception:
            pass


class Plan:
    """A graph compiled into a batched ciphertext program (host only; no GPU needed)."""

    def __init__(self, graph: Graph, params: Params | None = None, input_range=None,
                 margin_sigmas: float = 0.0, input_lens=None):
        import numpy as np
        self.params = default_params() if params is None else params
        if input_range is None:
            bits = graph.info()["input_bits"]
            input_range = (0, (1 << bits) - 1)
        lens = None
        if input_lens is not None:
            lens = np.ascontiguousarray(np.asarray(input_lens, dtype=np.int64))
        h = C.c_void_p()
        _check("pnb_plan_create",
               lib().pnb_plan_create(graph._h, C.byref(self.params),
                                     C.c_void_p(0) if lens is None else C.c_void_p(lens.ctypes.data),
                                     int(input_range[0]), int(input_range[1]),
                                     float(margin_sigmas), C.byref(h)))
        self._h = h
        s = _PlanSummary()
        _check("pnb_plan_info", lib().pnb_plan_info(h, C.byref(s)))
        self.input_elems = s.input_elems
        self.output_elems = s.output_elems
        self.pbs_per_sample = s.pbs_per_sample
        self.cost_per_sample = s.cost_per_sample
        self.num_instructions = s.num_instructions
        self.inputs = [self._tensor(0, i) for i in range(s.num_inputs)]
        self.outputs = [self._tensor(1, i) for i in range(s.num_outputs)]

    def _init_from_handle(self, h, params: Params):
        self.params = params
        self._h = h
        s = _PlanSummary()
        _check("pnb_plan_info", lib().pnb_plan_info(h, C.byref(s)))
        self.input_elems = s.input_elems
        self.output_elems = s.output_elems
        self.pbs_per_sample = s.pbs_per_sample
        self.cost_per_sample = s.cost_per_sample
        self.num_instructions = s.num_instructions
        self.inputs = [self._tensor(0, i) for i in range(s.num_inputs)]
        self.outputs = [self._tensor(1, i) for i in range(s.num_outputs)]

    def desc(self, is_output: bool, idx: int = 0) -> "TensorDesc":
        d = TensorDesc()
        _check("pnb_plan_tensor_desc",
               lib().pnb_plan_tensor_desc(self._h, int(is_output), idx, C.byref(d)))
        return d

    def _tensor(self, is_out, i):
        e, sc, lo, hi = C.c_int64(), C.c_int(), C.c_int64(), C.c_int64()
        _check("pnb_plan_tensor", lib().pnb_plan_tensor(self._h, is_out, i, C.byref(e),
                                                        C.byref(sc), C.byref(lo), C.byref(hi)))
        return {"elems": e.value, "scale": sc.value, "lo": lo.value, "hi": hi.value}

    def key_sets(self) -> list[tuple[int, int, int]]:
        """(base_log, levels, bootstraps per sample) of every key set the program uses."""
        n = lib().pnb_plan_key_sets(self._h, 0, None, None, None)
        b, l, c = (C.c_int * n)(), (C.c_int * n)(), (C.c_int64 * n)()
        lib().pnb_plan_key_sets(self._h, n, b, l, c)
        return [(b[i], l[i], c[i]) for i in range(n)]

    def report(self) -> str:
        n = lib().pnb_plan_report(self._h, None, 0)
        buf = C.create_string_buffer(n)
        lib().pnb_plan_report(self._h, buf, n)
        return buf.value.decode()

    def simulate(self, x):
        """Noise-free host execution on integers [batch][input_elems] -> (outputs, margin)."""
        import numpy as np
        x = np.ascontiguousarray(np.asarray(x, dtype=np.int64).reshape(-1, self.input_elems))
        y = np.zeros((x.shape[0], self.output_elems), dtype=np.int64)
        m = C.c_double()
        _check("pnb_plan_simulate",
               lib().pnb_plan_simulate(self._h, C.c_void_p(x.ctypes.data), x.shape[0],
                                       C.c_void_p(y.ctypes.data), C.byref(m)))
        return y, m.value

    def __del__(self):
        try:
            if self._h:
                lib().pnb_plan_free(self._h)
                self._h = None
        except Exception:
            pass


class Evaluator:
    """A plan bound to one GPU with its key sets (``EvalCtx`` + ``evaluate_graph``)."""

    def __init__(self, plan: Plan, device: int = 0, seed: int = 0, max_bytes: int = 0,
                 ring: "KeyRing | None" = None):
        self.plan = plan
        self.device = device if ring is None else ring.device
        self._ring = ring  # a borrowing evaluator keeps its ring alive
        h = C.c_void_p()
        if ring is None:
            _check("pnb_evaluator_create",
                   lib().pnb_evaluator_create(plan._h, device, seed, max_bytes, C.byref(h)))
        else:
            _check("pnb_evaluator_create_with",
                   lib().pnb_evaluator_create_with(plan._h, ring._h, max_bytes, C.byref(h)))
        self._h = h
        k = C.c_void_p()
        _check("pnb_evaluator_keys", lib().pnb_evaluator_keys(h, C.byref(k)))
        self.keys = KeySet(k, plan.params, self.device, seed, owner=self)
        self.row = plan.params.k * plan.params.N + 1

    def reserve(self, batch: int):
        """Allocate the ciphertext buffers for batches of up to ``batch`` samples now."""
        _check("pnb_evaluator_reserve", lib().pnb_evaluator_reserve(self._h, batch))

    def encrypt(self, x, seed: int = 1, first_index: int = 0) -> torch.Tensor:
        """Encrypt integers [batch][input_elems] at each input tensor's scale."""
        dev = torch.device("cuda", self.device)
        x = torch.as_tensor(x, dtype=torch.int64).reshape(-1, self.plan.input_elems)
        B = x.shape[0]
        ct = torch.empty((B, self.plan.input_elems, self.row), dtype=torch.int64, device=dev)
        off = 0
        for t in self.plan.inputs:
            e = t["elems"]
            part = encrypt(self.keys, x[:, off:off + e].reshape(-1), seed,
                           first_index + off * B, delta=1 << t["scale"])
            ct[:, off:off + e] = part.reshape(B, e, self.row)
            off += e
        return ct

    def evaluate(self, ct: torch.Tensor) -> torch.Tensor:
        ct = _u64(ct).contiguous()
        B = ct.numel() // (self.plan.input_elems * self.row)
        out = torch.empty((B, self.plan.output_elems, self.row), dtype=torch.int64,
                          device=ct.device)
        _check("pnb_evaluate", lib().pnb_evaluate(self._h, _ptr(ct), B, _ptr(out),
                                                  _stream(ct.device)))
        return out

    def decrypt(self, out: torch.Tensor) -> torch.Tensor:
        """Decode [batch][output_elems] signed integers at each output tensor's scale."""
        B = out.shape[0]
        ph = phase(self.keys, out.reshape(-1, self.row)).reshape(B, self.plan.output_elems)
        res = torch.empty_like(ph)
        off = 0
        for t in self.plan.outputs:
            e, s = t["elems"], t["scale"]
            res[:, off:off + e] = torch.bitwise_right_shift(ph[:, off:off + e] + (1 << (s - 1)), s)
            off += e
        return res

    def __del__(self):
        try:
            if self._h:
                lib().pnb_evaluator_free(self._h)
                self._h = None
        except Exception:
            pass


# ---- multi-GPU sharding ----------------------------------------------------------------------

def shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Samples [start, stop) of ``rank`` when ``batch`` samples are split over ``world`` ranks
    (contiguous, sizes differing by at most one)."""
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class Comm:
    """The library's NCCL communicator (``pnb_comm``) for the output all-gather of
    sample-sharded evaluation.  Every rank creates one with the same 128-byte id: draw it on one
    rank with ``Comm.unique_id()`` and hand it over out of band, or let ``from_process_group``
    broadcast it through an initialised ``torch.distributed`` group.  Close it explicitly
    (``close``, or ``abort`` after a peer failed); it is also a context manager."""

    def __init__(self, device: int, world: int, rank: int, uid: bytes):
        if len(uid) != 128:
            raise ValueError("a communicator id is 128 bytes")
        buf = C.create_string_buffer(bytes(uid), 128)
        h = C.c_void_p()
        _check("pnb_comm_create", lib().pnb_comm_create(int(device), int(world), int(rank),
                                                        buf, C.byref(h)))
        self.handle, self.device, self.world, self.rank = h, int(device), int(world), int(rank)

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        _check("pnb_comm_unique_id", lib().pnb_comm_unique_id(buf))
        return buf.raw

    @classmethod
    def from_process_group(cls, device: int, group=None) -> "Comm":
        import torch.distributed as dist
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        box = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        return cls(device, world, rank, box[0])

    def status(self):
        """Raise LibraryError if a collective of this communicator hit an asynchronous error."""
        _check("pnb_comm_status", lib().pnb_comm_status(self.handle))

    def allgather(self, local: torch.Tensor, batch: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's shard ``local`` (rows ``shard(batch, world, rank)``, any trailing shape)
        -> the full ``batch`` rows on every rank, enqueued on the current stream."""
        a, b = shard(batch, self.world, self.rank)
        if local.shape[0] != b - a:
            raise ValueError(f"rank {self.rank} holds {local.shape[0]} rows, its shard is {b - a}")
        row = tuple(local.shape[1:])
        row_bytes = math.prod(row) * local.element_size()
        if row_bytes == 0 or row_bytes % 8:
            raise ValueError("rows must be a whole, non-zero number of 64-bit words")
        if out is None:
            out = torch.empty((batch,) + row, dtype=local.dtype, device=local.device)
        local = local.contiguous()
        dev = torch.device("cuda", self.device)
        _check("pnb_allgather", lib().pnb_allgather(self.handle, _ptr(local if b > a else None),
                                                    _ptr(out), batch, row_bytes // 8,
                                                    _stream(dev)))
        return out

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            _check("pnb_comm_free", lib().pnb_comm_free(h))

    def abort(self):
        if self.handle:
            h, self.handle = self.handle, None
            _check("pnb_comm_abort", lib().pnb_comm_abort(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def shard_native(batch: int, world: int, rank: int) -> tuple[int, int]:
    """``shard`` as the library computes it (``pnb_shard``)."""
    a, b = C.c_int64(), C.c_int64()
    _check("pnb_shard", lib().pnb_shard(batch, world, rank, C.byref(a), C.byref(b)))
    return a.value, b.value


def gather_shards(local: torch.Tensor, batch: int, group=None,
                  comm: Comm | None = None) -> torch.Tensor:
    """All-gather per-rank shards (dim 0 = samples of ``shard(batch, world, rank)``) into the
    full batch on every rank.  With ``comm`` the library's own collective runs
    (``pnb_allgather``); otherwise ``torch.distributed`` does, the shards padded to the
    largest size (NCCL on GPU tensors, gloo on CPU tensors) and trimmed afterwards."""
    if comm is not None:
        return comm.allgather(local, batch)
    import torch.distributed as dist
    world = dist.get_world_size(group)
    sizes = [shard(batch, world, r) for r in range(world)]
    cap = max(b - a for a, b in sizes)
    buf = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    out = torch.empty((world * cap,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out, buf, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), buf, group=group)
    parts = [out[r * cap: r * cap + (b - a)] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts)


def evaluate_sharded(ev: "Evaluator", ct_all: torch.Tensor, group=None,
                     comm: Comm | None = None) -> torch.Tensor:
    """Strong-scaled evaluation: every rank evaluates its contiguous shard of the batch
    ``ct_all`` [batch][input_elems][kN+1] on its own GPU (identical key replicas from the same
    seed), then one all-gather (the library's, given ``comm``) reassembles the output
    ciphertexts on every rank."""
    if comm is not None:
        world, rank = comm.world, comm.rank
    else:
        import torch.distributed as dist
        world, rank = dist.get_world_size(group), dist.get_rank(group)
    a, b = shard(ct_all.shape[0], world, rank)
    local = ev.evaluate(ct_all[a:b].contiguous()) if b > a else torch.empty(
        (0, ev.plan.output_elems, ev.row), dtype=torch.int64, device=ct_all.device)
    return gather_shards(local, ct_all.shape[0], group, comm)


# ---- one op at a time ----------------------------------------------------------------------

class TensorDesc(C.Structure):
    """``pnb_tensor_desc``: elements per sample, value range, plaintext scale, noise."""
    _fields_ = [("elems", C.c_int64), ("lo", C.c_int64), ("hi", C.c_int64),
                ("scale_log2", C.c_int32), ("reserved", C.c_int32), ("log2_sigma", C.c_double)]

    @classmethod
    def make(cls, elems: int, lo: int, hi: int, scale_log2: int = 0, log2_sigma: float = 0.0):
        return cls(elems, lo, hi, scale_log2, 0, log2_sigma)

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_ if f != "reserved"}


class KeyRing:
    """Every key set the exact op programs may bootstrap with, from one seed on one GPU
    (``pnb_keyring``); ``keys`` is the client set that encrypts and decrypts."""

    def __init__(self, params: Params | None = None, seed: int = 0, device: int = 0):
        self.params = default_params() if params is None else params
        self.device = device
        h = C.c_void_p()
        _check("pnb_keyring_create",
               lib().pnb_keyring_create(device, C.byref(self.params), seed, C.byref(h)))
        self._h = h
        k = C.c_void_p()
        _check("pnb_keyring_keys", lib().pnb_keyring_keys(h, 0, C.byref(k)))
        self.keys = KeySet(k, self.params, device, seed, owner=self)
        self.row = self.params.k * self.params.N + 1

    def encrypt(self, values, scale_log2: int, seed: int, first_index: int = 0) -> torch.Tensor:
        """Encrypt integers (any shape [batch, elems]) at 2^scale_log2."""
        v = torch.as_tensor(values, dtype=torch.int64)
        ct = encrypt(self.keys, v.reshape(-1), seed, first_index, delta=1 << scale_log2)
        return ct.reshape(tuple(v.shape) + (self.row,))

    def decrypt(self, ct: torch.Tensor, scale_log2: int) -> torch.Tensor:
        """Signed rounding of every ciphertext's phase at 2^scale_log2."""
        ph = phase(self.keys, ct.reshape(-1, self.row)).reshape(ct.shape[:-1])
        return torch.bitwise_right_shift(ph + (1 << (scale_log2 - 1)), scale_log2)

    def __del__(self):
        try:
            if self._h:
                lib().pnb_keyring_free(self._h)
                self._h = None
        except Exception:
            pass


def op_plan(op: dict, inputs: list[TensorDesc], params: Params | None = None,
            out_scale: int = 0, out_sigma: float = 0.0, margin_sigmas: float = 0.0) -> Plan:
    """Compile one IR op over described inputs (``pnb_op_plan_create``) into a ``Plan``."""
    import json as _json
    params = default_params() if params is None else params
    text = _json.dumps(op).encode()
    arr = (TensorDesc * len(inputs))(*inputs)
    h = C.c_void_p()
    _check("pnb_op_plan_create",
           lib().pnb_op_plan_create(text, len(text), C.byref(params), C.cast(arr, C.c_void_p),
                                    len(inputs), out_scale, out_sigma, margin_sigmas,
                                    C.byref(h)))
    pl = Plan.__new__(Plan)
    pl._init_from_handle(h, params)
    return pl


def radix_plan(num_blocks: int, wide: TensorDesc, to_blocks: bool, signed: bool = True,
               block_max: int = 0, params: Params | None = None,
               margin_sigmas: float = 0.0) -> Plan:
    """Radix split (``to_blocks``) or merge program (``pnb_radix_plan_create``)."""
    params = default_params() if params is None else params
    h = C.c_void_p()
    _check("pnb_radix_plan_create",
           lib().pnb_radix_plan_create(C.byref(params), num_blocks, int(bool(signed)),
                                       int(bool(to_blocks)), block_max, C.byref(wide),
                                       margin_sigmas, C.byref(h)))
    pl = Plan.__new__(Plan)
    pl._init_from_handle(h, params)
    return pl


def _op_call(fn: str, ring: KeyRing, args_before, descs, tensors, out_elems: int,
             out_scale: int, out_sigma: float, out: torch.Tensor | None):
    batch = tensors[0].shape[0]
    dev = tensors[0].device
    if out is None:
        out = torch.empty((batch, out_elems, ring.row), dtype=torch.int64, device=dev)
    od = TensorDesc()
    ptrs = []
    for d, t in zip(descs, tensors):
        if t.shape[1] != d.elems or t.shape[2] != ring.row:
            raise ValueError(f"tensor of shape {tuple(t.shape)} does not match its descriptor "
                             f"({d.elems} elements of {ring.row} words)")
        ptrs += [C.byref(d), _ptr(_u64(t).contiguous())]
    _check(fn, getattr(lib(), fn)(ring._h, *args_before, *ptrs, batch, out_scale,
                                  C.c_double(out_sigma), _ptr(out), C.byref(od), _stream(dev)))
    return out, od


def requant_batch(ring: KeyRing, x: torch.Tensor, desc: TensorDesc, shift, mult=1,
                  round_bias=0, out_bits: int = 2, clamp_lut=None, channel_size: int = 0,
                  out_scale: int = 0, out_sigma: float = 0.0, out: torch.Tensor | None = None):
    """Exact Requant of wide ciphertexts ``x`` [batch, elems, kN+1] (``pnb_requant_batch``);
    ``shift``/``mult``/``round_bias`` are scalars (per-tensor) or per-channel sequences.
    Returns (output ciphertexts, output TensorDesc)."""
    import numpy as np
    sh = np.atleast_1d(np.asarray(shift, dtype=np.uint32))
    mu = np.atleast_1d(np.asarray(mult, dtype=np.uint64))
    rb = np.atleast_1d(np.asarray(round_bias, dtype=np.uint64))
    ch = len(sh)
    if len(mu) != ch or len(rb) != ch:
        raise ValueError("shift, mult and round_bias need one entry per channel")
    lut = None if clamp_lut is None else np.ascontiguousarray(clamp_lut, dtype=np.uint64)

    class Spec(C.Structure):
        _fields_ = [("channels", C.c_int32), ("out_bits", C.c_int32),
                    ("channel_size", C.c_int64), ("mult", C.c_void_p),
                    ("round_bias", C.c_void_p), ("shift", C.c_void_p),
                    ("clamp_lut", C.c_void_p)]

    spec = Spec(ch, out_bits, channel_size, mu.ctypes.data, rb.ctypes.data, sh.ctypes.data,
                None if lut is None else lut.ctypes.data)
    return _op_call("pnb_requant_batch", ring, [C.byref(spec)], [desc], [x], desc.elems,
                    out_scale, out_sigma, out)


def argmax_batch(ring: KeyRing, x: torch.Tensor, desc: TensorDesc, threshold: int,
                 out_scale: int = 0, out_sigma: float = 0.0, out: torch.Tensor | None = None):
    """[v >= threshold] of a one-element tensor per sample (``pnb_argmax_batch``)."""
    return _op_call("pnb_argmax_batch", ring, [C.c_int64(threshold)], [desc], [x], 1,
                    out_scale, out_sigma, out)


def add_batch(ring: KeyRing, a: torch.Tensor, da: TensorDesc, b: torch.Tensor, db: TensorDesc,
              out_scale: int = 0, out_sigma: float = 0.0, out: torch.Tensor | None = None):
    """a + b element-wise for tensors at one scale (``pnb_add_batch``)."""
    return _op_call("pnb_add_batch", ring, [], [da, db], [a, b], da.elems, out_scale,
                    out_sigma, out)
