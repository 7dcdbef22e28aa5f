"""Python binding of libsixi_smp.so, the C ABI of the B200 logits-to-token path.

The library is the product; this module only declares its entry points for ctypes and offers a
thin convenience layer over torch CUDA tensors (torch supplies device memory and streams). There
is no fallback: importing fails loudly when the library has not been built.

Entry points mirror the engine's sampler/verifier interface (include/sixi_smp.h):
  sample           DeterministicSampler::sample_token          src/core/core_execution.cpp:603-619
  candidates       DeterministicSampler::compute_sampling_candidates  (:449-584)
  greedy_argmax    DeterministicSampler::sample_greedy_argmax  (:394-407)
  verify           SpeculativeDecoder::step verification       src/speculative/speculative.cpp:589-916
and the device-side producer of JSON-object grammar masks (include/sixi_json.h, json_grammar.py).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("SIXI_SMP_LIB", _PKG / "lib" / "libsixi_smp.so"))

# status codes (ErrorCode values of the engine)
OK = 0
INVALID_ARGUMENT = 1
OUT_OF_BOUNDS = 2
OUT_OF_MEMORY_VRAM = 11
NUMERIC_NAN_OR_INF = 16
BACKEND_ERROR = 23
UNSUPPORTED_HARDWARE = 24

F32 = 0
BF16 = 1
STRICT_REPLAY = 0
ADAPTIVE = 1
ROW_MASKED = 1

PARAMS_DTYPE = np.dtype(
    [
        ("temperature", "<f4"),
        ("top_k", "<i4"),
        ("top_p", "<f4"),
        ("min_p", "<f4"),
        ("repetition_penalty", "<f4"),
        ("presence_penalty", "<f4"),
        ("frequency_penalty", "<f4"),
        ("mode", "<u4"),
        ("flags", "<u4"),
        ("reserved", "<u4"),
        ("seed", "<u8"),
        ("counter", "<u8"),
    ],
    align=True,
)
assert PARAMS_DTYPE.itemsize == 56

NUMERIC_FAIL = 0   # SIXI_SMP_NUMERIC_FAIL (NumericPolicy::FailAndInvalidate)
NUMERIC_CLAMP = 1  # SIXI_SMP_NUMERIC_CLAMP (NumericPolicy::EmergencyClampAndReport)
NUMERIC_REPORT_DTYPE = np.dtype(
    [
        ("healthy", "u1"),
        ("request_corrupted", "u1"),
        ("state_invalidated", "u1"),
        ("emergency_clamped", "u1"),
        ("status", "<i4"),
        ("nan_count", "<u8"),
        ("inf_count", "<u8"),
        ("first_bad_index", "<i8"),
    ]
)
assert NUMERIC_REPORT_DTYPE.itemsize == 32


class Rows(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_uint32),
        ("n_rows", ctypes.c_uint32),
        ("row_stride", ctypes.c_uint64),
    ]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64

# name -> (restype, argtypes); every symbol declared in include/sixi_smp.h
SIGNATURES = {
    "sixi_smp_create": (_I32, [_I32, _U32, _U32, ctypes.POINTER(_P)]),
    "sixi_smp_destroy": (_I32, [_P]),
    "sixi_smp_vocab": (_U32, [_P]),
    "sixi_smp_mask_words": (_U32, [_P]),
    "sixi_smp_status_string": (ctypes.c_char_p, [_I32]),
    "sixi_smp_sample": (_I32, [_P, ctypes.POINTER(Rows), _P, _P, _P, _P, _P, _U64, _P, _P, _P]),
    "sixi_smp_sample_host": (_I32, [_P, _P, _U32, _U32, _U64, _P, _P, _P, _P, _P, _U64, _P, _P, _P]),
    "sixi_smp_sample_host_async": (_I32, [_P, _P, _U32, _U32, _U64, _P, _P, _P, _P, _P, _U64, _P, _P, _P]),
    "sixi_smp_sample_indexed": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _U64, _P, _P, _P]),
    "sixi_smp_gather_rows": (_I32, [_P, _P, _P, _U32, _U32, _P, _U64, _P]),
    "sixi_smp_greedy_argmax": (_I32, [_P, ctypes.POINTER(Rows), _P, _P, _P, _P]),
    "sixi_smp_candidates": (_I32, [_P, ctypes.POINTER(Rows), _P, _P, _P, _P, _U32, _P, _P, _P, _P, _P]),
    "sixi_smp_verify": (_I32, [_P, ctypes.POINTER(Rows), _P, _P, _P, _U32, _U32, _P, _P, _P, _P, _P,
                               _U64, _P, _P, _P, _P, _P, _P, _P]),
    "sixi_smp_full_distribution": (_I32, [_P, ctypes.POINTER(Rows), _P, _P, _U64, _P]),
    "sixi_smp_numeric_policy": (_I32, [_P, _P, _U32, _U64, _U32, ctypes.c_float, _P, _P]),
    "sixi_smp_suffix_draft": (_I32, [_P, _P, _P, _U32, _U32, _U32, _P, _U32, _P, _P, _P]),
    "sixi_smp_verify_draft_logits": (_I32, [_P, ctypes.POINTER(Rows), ctypes.POINTER(Rows), _P, _P, _P, _U32, _U32,
                                            _P, _P, _P, _P, _P, _U64, _P, _P, _P, _P, _P, _P, _P]),
    "sixi_smp_verify_static": (_I32, [_I32, _U32, ctypes.POINTER(Rows), _P, _P, _P, _U32, _U32, _P, _P, _P,
                                      _P, _P, _U64, _P, _P, _P, _P, _P, _P, _P]),
    "sixi_smp_shard_candidates": (_I32, [_P, ctypes.POINTER(Rows), _U32, _U32, _U32, _P, _P, _P, _P, _U32,
                                         _P, _P, _P]),
    "sixi_smp_merge_shards": (_I32, [_P, _U32, _U32, _U32, _P, _P, _P, _P, _U64, _P, _P, _P]),
    "sixi_smp_philox_uniform": (ctypes.c_double, [_U64, _U64, _U32]),
    # include/sixi_json.h: the device-side grammar-mask producer (sixi_smp.json_grammar)
    "sixi_json_vocab_create": (_I32, [_I32, _P, _P, _U32, _P, _I32, ctypes.POINTER(_P)]),
    "sixi_json_vocab_destroy": (None, [_P]),
    "sixi_json_vocab_size": (_U32, [_P]),
    "sixi_json_reset": (_I32, [_P, _P, _U32, _P]),
    "sixi_json_fill_masks": (_I32, [_P, _P, _U32, _P, _U64, _P]),
    "sixi_json_advance": (_I32, [_P, _P, _U32, _P, _U64, _P, _P, _P]),
    "sixi_json_expand_drafts": (_I32, [_P, _P, _U32, _P, _U32, _P, _P, _P]),
    # json_schema grammar masks (include/sixi_schema.h)
    "sixi_schema_compile": (_I32, [_I32, _P, ctypes.c_size_t, _P, _P, _U32, _P, _I32, _P, ctypes.c_size_t,
                                   ctypes.POINTER(_P)]),
    "sixi_schema_destroy": (None, [_P]),
    "sixi_schema_vocab_size": (_U32, [_P]),
    "sixi_schema_reset": (_I32, [_P, _P, _U32, _P]),
    "sixi_schema_fill_masks": (_I32, [_P, _P, _U32, _P, _U64, _P]),
    "sixi_schema_advance": (_I32, [_P, _P, _U32, _P, _U64, _P, _P, _P]),
    "sixi_schema_check_text": (_I32, [_P, _P, ctypes.c_size_t]),
}


def load(path: Path | str = LIB_PATH) -> ctypes.CDLL:
    path = Path(path)
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python sixi-asi_b200/build_lib.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def _lib() -> ctypes.CDLL:
    """The loaded library (loaded on first use; raises ImportError when it is not built)."""
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def status_string(st: int) -> str:
    return _lib().sixi_smp_status_string(int(st)).decode()


def philox_uniform(seed: int, counter: int, slot: int) -> float:
    return float(_lib().sixi_smp_philox_uniform(seed, counter, slot))


class SixiError(RuntimeError):
    def __init__(self, where: str, status: int):
        super().__init__(f"{where}: {status_string(status)} ({status})")
        self.status = status


def _check(where: str, st: int) -> None:
    if st != OK:
        raise SixiError(where, st)


def make_params(n: int, **fields) -> np.ndarray:
    """Array of n parameter records; scalars or per-row arrays for any field."""
    p = np.zeros(n, dtype=PARAMS_DTYPE)
    p["top_p"] = 1.0
    p["repetition_penalty"] = 1.0
    p["mode"] = ADAPTIVE
    for k, v in fields.items():
        p[k] = v
    return p


def _ptr(t) -> int:
    """Device pointer of a torch tensor, or 0 for None."""
    return 0 if t is None else int(t.data_ptr())


class Sampler:
    """A handle bound to one device and vocabulary (sixi_smp_create)."""

    def __init__(self, device: int, max_rows: int, vocab: int):
        h = _P()
        _check("sixi_smp_create", _lib().sixi_smp_create(device, max_rows, vocab, ctypes.byref(h)))
        self.h = h
        self.device = device
        self.vocab = vocab
        self.max_rows = max_rows
        self.mask_words = int(_lib().sixi_smp_mask_words(h))

    def close(self) -> None:
        if self.h:
            _lib().sixi_smp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- device-pointer entry points (torch tensors on this device) ---------------------------
    @staticmethod
    def _rows(logits) -> Rows:
        import torch

        dt = {torch.float32: F32, torch.bfloat16: BF16}[logits.dtype]
        assert logits.dim() == 2 and logits.stride(1) == 1
        return Rows(logits.data_ptr(), dt, logits.shape[0], logits.stride(0))

    @staticmethod
    def _stream(stream) -> int:
        import torch

        s = stream if stream is not None else torch.cuda.current_stream()
        return int(s.cuda_stream)

    def sample(self, logits, params, masks=None, hist=None, hist_off=None, uniforms=None, step=0,
               out_tokens=None, out_status=None, stream=None):
        import torch

        n = logits.shape[0]
        dev = logits.device
        if out_tokens is None:
            out_tokens = torch.empty(n, dtype=torch.int32, device=dev)
        if out_status is None:
            out_status = torch.empty(n, dtype=torch.int32, device=dev)
        rows = self._rows(logits)
        st = _lib().sixi_smp_sample(self.h, ctypes.byref(rows), _ptr(params), _ptr(masks), _ptr(hist),
                                 _ptr(hist_off), _ptr(uniforms), step, _ptr(out_tokens),
                                 _ptr(out_status), self._stream(stream))
        _check("sixi_smp_sample", st)
        return out_tokens, out_status

    def sample_indexed(self, logits, row_map, params, out_tokens, out_status, masks=None, hist=None, hist_off=None,
                       uniforms=None, step=0, stream=None):
        """sixi_smp_sample_indexed: row j of `logits` sampled as batch row row_map[j] (int32 device
        tensor); params / masks / hist / uniforms / outputs are the whole batch's."""
        rows = self._rows(logits)
        st = _lib().sixi_smp_sample_indexed(self.h, ctypes.byref(rows), _ptr(row_map), _ptr(params), _ptr(masks),
                                            _ptr(hist), _ptr(hist_off), _ptr(uniforms), step, _ptr(out_tokens),
                                            _ptr(out_status), self._stream(stream))
        _check("sixi_smp_sample_indexed", st)
        return out_tokens, out_status

    def gather_rows(self, src, row_index, width: int, out=None, stream=None):
        """sixi_smp_gather_rows: out[j, :width] = src[row_index[j], :width] (device tensors)."""
        import torch

        n = int(row_index.numel())
        if out is None:
            out = torch.empty((n, width), dtype=src.dtype, device=src.device)
        rows = self._rows(src)
        st = _lib().sixi_smp_gather_rows(self.h, ctypes.byref(rows), _ptr(row_index), n, width, _ptr(out),
                                         out.stride(0), self._stream(stream))
        _check("sixi_smp_gather_rows", st)
        return out

    def greedy_argmax(self, logits, masks=None, stream=None):
        import torch

        n = logits.shape[0]
        tok = torch.empty(n, dtype=torch.int32, device=logits.device)
        sts = torch.empty(n, dtype=torch.int32, device=logits.device)
        rows = self._rows(logits)
        st = _lib().sixi_smp_greedy_argmax(self.h, ctypes.byref(rows), _ptr(masks), _ptr(tok), _ptr(sts),
                                        self._stream(stream))
        _check("sixi_smp_greedy_argmax", st)
        return tok, sts

    def candidates(self, logits, params, max_out=256, masks=None, hist=None, hist_off=None,
                   stream=None):
        import torch

        n = logits.shape[0]
        dev = logits.device
        ids = torch.full((n, max_out), -1, dtype=torch.int32, device=dev)
        probs = torch.zeros((n, max_out), dtype=torch.float64, device=dev)
        cnt = torch.zeros(n, dtype=torch.int32, device=dev)
        sts = torch.empty(n, dtype=torch.int32, device=dev)
        rows = self._rows(logits)
        st = _lib().sixi_smp_candidates(self.h, ctypes.byref(rows), _ptr(params), _ptr(masks), _ptr(hist),
                                     _ptr(hist_off), max_out, _ptr(ids), _ptr(probs), _ptr(cnt),
                                     _ptr(sts), self._stream(stream))
        _check("sixi_smp_candidates", st)
        return ids, probs, cnt, sts

    def verify(self, target, drafts, params, draft_probs=None, n_drafts=None, masks=None, hist=None,
               hist_off=None, uniforms=None, step=0, stream=None):
        import torch

        S, k = drafts.shape
        dev = target.device
        acc = torch.empty(S, dtype=torch.int32, device=dev)
        toks = torch.empty((S, k + 1), dtype=torch.int32, device=dev)
        ntok = torch.empty(S, dtype=torch.int32, device=dev)
        frej = torch.empty(S, dtype=torch.int32, device=dev)
        used = torch.empty(S, dtype=torch.int32, device=dev)
        sts = torch.empty(S, dtype=torch.int32, device=dev)
        rows = self._rows(target)
        st = _lib().sixi_smp_verify(self.h, ctypes.byref(rows), _ptr(draft_probs), _ptr(drafts),
                                 _ptr(n_drafts), S, k, _ptr(params), _ptr(masks), _ptr(hist),
                                 _ptr(hist_off), _ptr(uniforms), step, _ptr(acc), _ptr(toks), _ptr(ntok),
                                 _ptr(frej), _ptr(used), _ptr(sts), self._stream(stream))
        _check("sixi_smp_verify", st)
        return dict(accepted=acc, tokens=toks, n_tokens=ntok, first_reject=frej, uniforms_used=used,
                    status=sts)

    def verify_draft_logits(self, target, draft_logits, draft_temperatures, drafts, params, n_drafts=None,
                            masks=None, hist=None, hist_off=None, uniforms=None, step=0, stream=None):
        """verify with q = full_distribution(draft_logits, draft_temperatures), never stored."""
        import torch

        S, k = drafts.shape
        dev = target.device
        acc = torch.empty(S, dtype=torch.int32, device=dev)
        toks = torch.empty((S, k + 1), dtype=torch.int32, device=dev)
        ntok = torch.empty(S, dtype=torch.int32, device=dev)
        frej = torch.empty(S, dtype=torch.int32, device=dev)
        used = torch.empty(S, dtype=torch.int32, device=dev)
        sts = torch.empty(S, dtype=torch.int32, device=dev)
        rows = self._rows(target)
        qrows = self._rows(draft_logits)
        st = _lib().sixi_smp_verify_draft_logits(
            self.h, ctypes.byref(rows), ctypes.byref(qrows), _ptr(draft_temperatures), _ptr(drafts), _ptr(n_drafts),
            S, k, _ptr(params), _ptr(masks), _ptr(hist), _ptr(hist_off), _ptr(uniforms), step, _ptr(acc),
            _ptr(toks), _ptr(ntok), _ptr(frej), _ptr(used), _ptr(sts), self._stream(stream))
        _check("sixi_smp_verify_draft_logits", st)
        return dict(accepted=acc, tokens=toks, n_tokens=ntok, first_reject=frej, uniforms_used=used,
                    status=sts)

    def full_distribution(self, logits, temperatures, stream=None):
        """compute_full_distribution per row: fp32 probabilities [n_rows, vocab]."""
        import torch

        out = torch.empty((logits.shape[0], self.vocab), dtype=torch.float32, device=logits.device)
        rows = self._rows(logits)
        st = _lib().sixi_smp_full_distribution(self.h, ctypes.byref(rows), _ptr(temperatures), _ptr(out),
                                            self.vocab, self._stream(stream))
        _check("sixi_smp_full_distribution", st)
        return out

    def numeric_policy(self, logits, policy: int = NUMERIC_FAIL, clamp_abs_max: float = 0.0, out=None, stream=None):
        """inspect_and_apply_numeric_policy per row of fp32 `logits` [n_rows, >= vocab] (a row view
        of wider rows is fine), in place under NUMERIC_CLAMP. Returns the reports as a uint8 device
        tensor [n_rows, 32] (numeric_reports() views them as NUMERIC_REPORT_DTYPE records)."""
        import torch

        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("numeric_policy takes fp32 rows [n_rows, >= vocab] with unit column stride")
        n = logits.shape[0]
        if out is None:
            out = torch.empty((n, 32), dtype=torch.uint8, device=logits.device)
        st = _lib().sixi_smp_numeric_policy(self.h, _ptr(logits), n, logits.stride(0), policy, clamp_abs_max,
                                            _ptr(out), self._stream(stream))
        _check("sixi_smp_numeric_policy", st)
        return out

    def suffix_draft(self, hist, hist_off, k: int = 8, min_match_len: int = 3, max_window_tokens: int = 16384,
                     anchors=None, out=None, out_match=None, stream=None):
        """SuffixDrafter::propose (or ::propose_anchored with `anchors` [n_streams]) for the CSR
        histories (hist int32, hist_off int64 [n_streams + 1], device tensors). Returns
        (drafts int32 [n_streams, k], match_len int32 [n_streams]; 0 and -1 drafts without a proposal)."""
        import torch

        n = hist_off.numel() - 1
        dev = hist_off.device
        if out is None:
            out = torch.empty((n, k), dtype=torch.int32, device=dev)
        if out_match is None:
            out_match = torch.empty(n, dtype=torch.int32, device=dev)
        st = _lib().sixi_smp_suffix_draft(self.h, _ptr(hist), _ptr(hist_off), n, min_match_len, max_window_tokens,
                                          _ptr(anchors), k, _ptr(out) if k else None, _ptr(out_match),
                                          self._stream(stream))
        _check("sixi_smp_suffix_draft", st)
        return out, out_match

    # -- vocab-sharded mode ----------------------------------------------------------------------
    def shard_candidates(self, shard_logits, vocab_offset: int, shard_vocab: int, params, top_n: int = 64,
                         masks=None, hist=None, hist_off=None, stream=None):
        """Stage 1 on this rank's slice: shard_logits [n_rows, >= shard_vocab] (a column slice of the
        full rows is fine). Returns (cand int32 [n_rows, top_n, 2] = (logit bits, id), stats uint8
        [n_rows, 24])."""
        import torch

        n = shard_logits.shape[0]
        cand = torch.empty((n, top_n, 2), dtype=torch.int32, device=shard_logits.device)
        stats = torch.empty((n, 24), dtype=torch.uint8, device=shard_logits.device)
        rows = self._rows(shard_logits)
        st = _lib().sixi_smp_shard_candidates(self.h, ctypes.byref(rows), vocab_offset, shard_vocab, self.vocab,
                                           _ptr(params), _ptr(masks), _ptr(hist), _ptr(hist_off), top_n,
                                           _ptr(cand), _ptr(stats), self._stream(stream))
        _check("sixi_smp_shard_candidates", st)
        return cand, stats

    def merge_shards(self, gathered_cand, gathered_stats, params, uniforms=None, step: int = 0, stream=None):
        """Stage 2: gathered_cand [n_shards, n_rows, top_n, 2], gathered_stats [n_shards, n_rows, 24]."""
        import torch

        S, n, top_n = gathered_cand.shape[0], gathered_cand.shape[1], gathered_cand.shape[2]
        tok = torch.empty(n, dtype=torch.int32, device=gathered_cand.device)
        sts = torch.empty(n, dtype=torch.int32, device=gathered_cand.device)
        st = _lib().sixi_smp_merge_shards(self.h, n, S, top_n, _ptr(gathered_cand), _ptr(gathered_stats),
                                       _ptr(params), _ptr(uniforms), step, _ptr(tok), _ptr(sts),
                                       self._stream(stream))
        _check("sixi_smp_merge_shards", st)
        return tok, sts

    # -- host-buffer entry point ---------------------------------------------------------------
    def sample_host(self, logits: np.ndarray, params: np.ndarray, masks=None, hist=None, hist_off=None,
                    uniforms=None, step=0, out_tokens=None, out_status=None, stream=None, wait: bool = True):
        """logits: host array [n, stride] (float32, or uint16 holding bf16). With wait=False the call
        is sixi_smp_sample_host_async: it returns once the work is queued, and the outputs are valid
        after `stream` is synchronised (host buffers pinned and kept unchanged until then)."""
        n = logits.shape[0]
        dt = BF16 if logits.dtype == np.uint16 else F32
        if out_tokens is None:
            out_tokens = np.empty(n, dtype=np.int32)
        if out_status is None:
            out_status = np.empty(n, dtype=np.int32)

        def hp(a):
            return 0 if a is None else a.ctypes.data

        fn = _lib().sixi_smp_sample_host if wait else _lib().sixi_smp_sample_host_async
        st = fn(self.h, hp(logits), dt, n, logits.shape[1], hp(params), hp(masks), hp(hist), hp(hist_off),
                hp(uniforms), step, hp(out_tokens), hp(out_status), self._stream(stream) if stream is not None else 0)
        _check("sixi_smp_sample_host" if wait else "sixi_smp_sample_host_async", st)
        return out_tokens, out_status


STATIC_VERIFY_ROWS = 4096  # SIXI_SMP_STATIC_VERIFY_ROWS


def verify_static(vocab: int, target, drafts, params, draft_probs=None, n_drafts=None, masks=None, hist=None,
                  hist_off=None, uniforms=None, step=0, stream=None):
    """sixi_smp_verify_static: the verifier without a handle or any allocation inside the call
    (its workspace is a static device array of STATIC_VERIFY_ROWS rows). Outputs are allocated
    here by torch, on the target's device."""
    import torch

    S, k = drafts.shape
    dev = target.device
    acc = torch.empty(S, dtype=torch.int32, device=dev)
    toks = torch.empty((S, k + 1), dtype=torch.int32, device=dev)
    ntok = torch.empty(S, dtype=torch.int32, device=dev)
    frej = torch.empty(S, dtype=torch.int32, device=dev)
    used = torch.empty(S, dtype=torch.int32, device=dev)
    sts = torch.empty(S, dtype=torch.int32, device=dev)
    rows = Sampler._rows(target)
    st = _lib().sixi_smp_verify_static(dev.index or 0, vocab, ctypes.byref(rows), _ptr(draft_probs), _ptr(drafts),
                                       _ptr(n_drafts), S, k, _ptr(params), _ptr(masks), _ptr(hist), _ptr(hist_off),
                                       _ptr(uniforms), step, _ptr(acc), _ptr(toks), _ptr(ntok), _ptr(frej),
                                       _ptr(used), _ptr(sts), Sampler._stream(stream))
    _check("sixi_smp_verify_static", st)
    return dict(accepted=acc, tokens=toks, n_tokens=ntok, first_reject=frej, uniforms_used=used, status=sts)


def numeric_reports(t) -> np.ndarray:
    """The uint8 [n_rows, 32] report tensor of Sampler.numeric_policy as NUMERIC_REPORT_DTYPE records."""
    return np.ascontiguousarray(t.cpu().numpy()).view(NUMERIC_REPORT_DTYPE).reshape(-1)
