"""``B200Executor``: the reference ``Executor`` surface over libqtts_b200.so.

Reference: engine/backend/executor.py:487-1612 (``Executor``), 357-480
(``GPUFuture`` / ``StepOutput``).  The engine loop calls the same methods
(``load``, ``prefill``, ``prefill_prefix_only``, ``prefill_from_prefix``,
``launch_decode_step`` -> ``GPUFuture.wait`` -> ``StepOutput``, ``warmup``,
``shutdown``; properties ``kv_pool``, ``max_batch_size``, ``max_seq_len``).

What changes underneath:

* KV is paged and written by the step itself, so ``StepOutput.batch_talker_kv``
  is ``None`` and the engine loop's delta scatter
  (engine/backend/engine_loop.py:2086-2092) has nothing to do.
* Per-slot decode state lives on the device, indexed by slot id: token counts,
  the next input embedding (``codec_sum + text`` computed by the step), the
  text embedding to add next, temperature / penalty and the Philox noise
  key / counter.  The reference keeps these as per-slot torch tensors and
  rebuilds batch inputs every step (executor.py:1259-1469).
* A decode step for a given batch size is captured once in a CUDA graph and
  replayed; the host only writes the slot list.
* Code2wav runs in the same step (and graph) as the talker, one frame per
  stream, like the fused plan (export_09_talker_code2wav_fused.py:145-160):
  ``audio_chunks`` carries each stream's 1920 fp32 samples as bytes
  (executor.py:424-435).  Its streaming state is device-resident per slot
  (``runtime/code2wav.py``), so ``make_zero_conv_states`` /
  ``make_zero_transconv_states`` return empty lists and a stream's decoder
  state is zeroed by the prefill that starts it.
"""

from __future__ import annotations

import hashlib
import logging
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch

from .. import _lib
from ..config import EngineConfig, PagedPoolConfig
from ..weights import make_code2wav_weights, make_cp_weights, make_talker_weights
from .code2wav import DeviceCode2Wav, warm_state_parts
from .model import DeviceModel
from .pool import PagedKVCachePool, PagedPrefixKVCache, SlotState

logger = logging.getLogger(__name__)

_MAX_SEED = (1 << 63) - 1


def stable_sampling_seed(base_seed: int, *parts: object) -> int:
    """Deterministic per-(session, segment) seed (executor.py:45-52)."""
    h = hashlib.blake2b(digest_size=16)
    h.update(str(int(base_seed)).encode("utf-8"))
    for part in parts:
        h.update(b"\0")
        h.update(str(part).encode("utf-8"))
    return int.from_bytes(h.digest()[:8], "little") & _MAX_SEED


@dataclass
class StepOutput:
    """Results of one decode step (executor.py:455-480)."""

    slots: List[SlotState]
    eos_flags: List[bool]
    audio_chunks: List[Optional[bytes]]
    batch_talker_kv: Optional[torch.Tensor] = None
    batch_c2w_kv: Optional[torch.Tensor] = None
    original_past_lens: List[int] = field(default_factory=list)
    padded_past_len: int = 0
    split_c2w_conv: List[list] = field(default_factory=list)
    split_c2w_transconv: List[list] = field(default_factory=list)
    codec_sum: Optional[torch.Tensor] = None
    full_codec: Optional[torch.Tensor] = None
    updated_tc: Optional[torch.Tensor] = None
    used_pingpong: bool = False
    step_input_embeds: Optional[torch.Tensor] = None


class BatchRows:
    """``StepOutput.codec_sum`` as the engine loop indexes it: row i of the step's batch,
    ``codec_sum[i:i+1]`` -> ``[1, 1, H]`` (engine_loop.py:2170-2197), read from the
    slot-indexed codec-sum buffer of the step's parity (valid until the step two launches
    later reuses it, i.e. while the loop processes this step's output)."""

    def __init__(self, buf: torch.Tensor, slot_ids: List[int]):
        self._buf = buf
        self._ids = slot_ids

    @property
    def dtype(self):
        return self._buf.dtype

    @property
    def device(self):
        return self._buf.device

    @property
    def shape(self):
        return (len(self._ids), 1, self._buf.shape[-1])

    def __len__(self):
        return len(self._ids)

    def __getitem__(self, key) -> torch.Tensor:
        if isinstance(key, int):
            return self._buf[self._ids[key]].view(1, -1)
        return self._buf[self._ids[key]].unsqueeze(1)

    def tensor(self) -> torch.Tensor:
        return self[:]


@dataclass
class GPUFuture:
    """Handle to an in-flight decode step (executor.py:357-452)."""

    _executor: Any = None
    _event: Any = None
    _slots: List[SlotState] = field(default_factory=list)
    _original_past_lens: List[int] = field(default_factory=list)
    _codes_host: Optional[torch.Tensor] = None
    _codes_dev: Optional[torch.Tensor] = None
    _codec_sum: Optional[BatchRows] = None
    _status_host: Optional[torch.Tensor] = None
    _wav_host: Optional[torch.Tensor] = None

    def wait(self) -> StepOutput:
        if self._event is not None:
            self._event.synchronize()
        n = len(self._slots)
        if self._status_host is not None and int(self._status_host[0]) != 0:
            st = int(self._status_host[0])
            _lib.check(st, "decode step scheduler")
        codes = self._codes_host[:n].clone() if self._codes_host is not None else None
        eos_id = self._executor._config.talker.codec_eos_id if self._executor else 2150
        eos = (codes[:, 0] == eos_id).tolist() if codes is not None else [False] * n
        if self._wav_host is not None:
            wav = self._wav_host[:n].numpy()  # one view of the pinned buffer, then a bytes copy per row
            audio = [wav[i].tobytes() for i in range(n)]
        else:
            audio = [None] * n
        return StepOutput(slots=self._slots, eos_flags=eos, audio_chunks=audio,
                          original_past_lens=self._original_past_lens, codec_sum=self._codec_sum,
                          full_codec=codes, split_c2w_conv=[[] for _ in range(n)],
                          split_c2w_transconv=[[] for _ in range(n)])


class B200Executor:
    """Drop-in for ``engine.backend.executor.Executor`` on a B200."""

    def __init__(self, *, engine_dir: str = "", weights_dir: str = "", device_id: int = 0,
                 max_batch_size: int = 64, max_seq_len: int = 1024, model_config: Optional[EngineConfig] = None,
                 do_sample: bool = False, temperature: float = 0.9, repetition_penalty: float = 1.05,
                 random_seed: int = 0, num_blocks: int = 8192, weights: Optional[Dict[str, torch.Tensor]] = None,
                 weight_seed: int = 1, max_prefill_rows: int = 512, use_cuda_graphs: bool = True,
                 enable_code2wav: bool = True, c2w_weights: Optional[Dict[str, torch.Tensor]] = None):
        if not torch.cuda.is_available():
            raise RuntimeError("B200Executor needs a CUDA device (no CPU path)")
        self._device = torch.device("cuda", device_id)
        self._config = model_config or EngineConfig()
        self._config.pool = PagedPoolConfig(block_size=16, num_blocks=num_blocks, max_slots=max_batch_size,
                                            max_seq_len=max_seq_len)
        self._max_batch = max_batch_size
        self._max_seq_len = max_seq_len
        self._max_input_len = max_prefill_rows
        self._do_sample = do_sample
        self._temperature = temperature
        self._repetition_penalty = repetition_penalty
        self._random_seed = int(random_seed)
        self._weights = weights
        self._weight_seed = weight_seed
        self._use_graphs = use_cuda_graphs
        self._enable_c2w = enable_code2wav
        self._c2w_weights = c2w_weights
        self._c2w: Optional[DeviceCode2Wav] = None
        # Two streams: talker + code predictor (latency-bound kernel chain, high priority)
        # and code2wav (low priority).  Code2wav of step t only needs step t's codes, so it
        # runs while step t + 1's talker and code predictor run.
        self._stream = torch.cuda.Stream(device=self._device, priority=-1)
        self._c2w_stream = torch.cuda.Stream(device=self._device, priority=0)
        self._model: Optional[DeviceModel] = None
        self._kv_pool: Optional[PagedKVCachePool] = None
        self._graphs: Dict[int, Any] = {}
        self._embedding_weights = None
        # decode steps alternate between two sets of step buffers (parity); the events of
        # the last step of each parity guard their reuse two steps later
        self._parity = 0
        self._done_a: List[Any] = [None, None]
        self._done_b: List[Any] = [None, None]
        self._c2w_warm: Dict[int, Any] = {}  # slot -> session whose warm code2wav state is installed

    # -- properties the engine loop reads ---------------------------------
    @property
    def kv_pool(self) -> PagedKVCachePool:
        return self._kv_pool

    @property
    def max_batch_size(self) -> int:
        return self._max_batch

    @property
    def max_seq_len(self) -> int:
        return self._max_seq_len

    @property
    def model(self) -> DeviceModel:
        return self._model

    # -- lifecycle --------------------------------------------------------
    def load(self) -> None:
        cfg = self._config
        W = self._weights
        if W is None:
            W = make_talker_weights(cfg.talker, self._weight_seed, device=self._device)
            W.update(make_cp_weights(cfg.cp, self._weight_seed, device=self._device))
        with torch.cuda.device(self._device):
            self._model = DeviceModel(cfg, W, self._device, max_batch=self._max_batch,
                                      max_prefill_rows=self._max_input_len)
            if self._enable_c2w:
                Wc = self._c2w_weights
                if Wc is None:
                    Wc = make_code2wav_weights(cfg.c2w, self._weight_seed, device=self._device)
                # one frame per decode step plus the prefill frame
                self._c2w = DeviceCode2Wav(cfg.c2w, Wc, self._device, max_slots=self._max_batch,
                                           max_frames=self._max_seq_len + 1)
                self._c2w.set_background(True)  # runs beside the next step's talker (stream B)
        self._weights = None
        self._c2w_weights = None
        self._alloc_state()
        self._kv_pool = PagedKVCachePool(self._model, self._max_batch)
        self._kv_pool.counts_reset_hook = self._reset_slot_state
        logger.info("B200Executor loaded (slots=%d, blocks=%d)", self._max_batch, cfg.pool.num_blocks)

    def make_prefix_cache(self, max_entries: int = 16, max_prefix_len: int = 512) -> PagedPrefixKVCache:
        return PagedPrefixKVCache(self._kv_pool, max_entries=max_entries, max_prefix_len=max_prefix_len)

    def set_embedding_weights(self, weights) -> None:
        self._embedding_weights = weights

    def shutdown(self) -> None:
        self._graphs.clear()
        if self._kv_pool is not None:
            self._kv_pool.close()
        if self._c2w is not None:
            self._c2w.close()
        self._c2w = None
        if self._model is not None:
            self._model.close()
        self._model = None
        self._kv_pool = None

    # -- code2wav state (device-resident per slot) -------------------------
    def make_zero_conv_states(self) -> list:
        """executor.py:701-706.  The conv states live on the device, per slot."""
        return []

    def make_zero_transconv_states(self) -> list:
        """executor.py:708-713.  The transposed-conv states live on the device, per slot."""
        return []

    def apply_c2w_warm_state(self, slot: SlotState, c2w_kv, conv_states, transconv_states, frame_idx: int) -> bool:
        """executor.py:715-757: install a warmed code2wav state (the reference's tensors: 2 x layers
        window KV as one [1, 2L, heads, T, head_dim] tensor, 17 conv states, 4 transposed-conv
        overlap tails) before the slot's first target frame.  The tensors are converted to this
        decoder's layout (``warm_state_parts``: the overlap tails back to the previous input row
        by least squares) and written into the slot's device state, ordered on the code2wav
        stream; the slot's next prefill then decodes its first frame from that state instead of
        from zero.  Returns False (state not applied, as the reference does on a mismatch) for
        missing tensors, wrong counts or shapes."""
        if c2w_kv is None or conv_states is None or transconv_states is None or self._c2w is None:
            return False
        if len(conv_states) != 17 or len(transconv_states) != 4:
            logger.warning("Skipping Code2Wav warm state: %d conv / %d transconv states (expected 17 / 4)",
                           len(conv_states), len(transconv_states))
            return False
        cur = torch.cuda.current_stream(self._device)
        try:
            with torch.cuda.stream(cur):
                parts = warm_state_parts(self._config.c2w, self._c2w.P, self._c2w.state_layout(), c2w_kv,
                                         conv_states, transconv_states, int(frame_idx), self._device,
                                         tail_qr=self._c2w.tail_qr)
        except ValueError as exc:
            logger.warning("Skipping Code2Wav warm state (slot=%d): %s", slot.slot_id, exc)
            return False
        b = self._c2w_stream  # every code2wav call runs on this stream, in order
        b.wait_stream(cur)
        for t in parts:
            t.record_stream(b)
        self._c2w.install_state(slot.slot_id, parts, max(0, int(frame_idx)), stream=b)
        slot.frame_idx = max(0, int(frame_idx))
        self._c2w_warm[slot.slot_id] = slot.session_id
        return True

    # -- per-slot device state --------------------------------------------
    def _alloc_state(self) -> None:
        t, c = self._config.talker, self._config.cp
        S, B, dev = self._max_batch, self._max_batch, self._device
        f32, i32, i64 = torch.float32, torch.int32, torch.int64
        self.counts = torch.zeros(S, t.codec_vocab_size, dtype=i64, device=dev)
        self.next_x = torch.zeros(S, t.hidden_size, dtype=f32, device=dev)
        self.text_add = torch.zeros(S, t.hidden_size, dtype=f32, device=dev)
        # codec sums by parity like the codes: the engine loop reads step t's while t + 1 runs
        self.codec_sum_buf = torch.zeros(3, S, t.hidden_size, dtype=f32, device=dev)
        self.codec_sum = self.codec_sum_buf[2]
        self.temperature = torch.ones(S, dtype=f32, device=dev)
        self.penalty = torch.full((S,), self._repetition_penalty, dtype=f32, device=dev)
        self.noise_key = torch.zeros(S, dtype=i64, device=dev)
        self.noise_step = torch.zeros(S, dtype=i32, device=dev)
        self.zero_gumbel = torch.zeros(B, t.logits_topk, dtype=f32, device=dev)
        self.zero_cp_gumbel = torch.zeros(B, c.num_stages, t.logits_topk, dtype=f32, device=dev)
        # step buffers by parity: [0], [1] alternate between decode steps, [2] serves prefill
        self.slots_buf = torch.zeros(3, B, dtype=i32, device=dev)
        self.slots_host_buf = torch.zeros(3, B, dtype=i32).pin_memory()
        self.slots_dev = self.slots_buf[2]
        self.slots_host = self.slots_host_buf[2]
        self.hidden = torch.zeros(B, t.hidden_size, dtype=torch.bfloat16, device=dev)
        self.logits = torch.zeros(B, t.codec_vocab_size, dtype=f32, device=dev)
        self.codes_buf = torch.zeros(3, B, 1 + c.num_stages, dtype=i64, device=dev)
        self.codes_host_buf = torch.zeros(3, B, 1 + c.num_stages, dtype=i64).pin_memory()
        self.codes = self.codes_buf[2]  # the last prefill's frame
        self.status = torch.zeros(1, dtype=i32, device=dev)
        self.status_host_buf = torch.zeros(3, 1, dtype=i32).pin_memory()
        self.status_host = self.status_host_buf[2]
        spf = self._config.c2w.samples_per_frame
        self.wav = torch.zeros(B, spf, dtype=f32, device=dev) if self._enable_c2w else None
        self.wav_host_buf = torch.zeros(3, B, spf, dtype=f32).pin_memory() if self._enable_c2w else None
        self.wav_host = self.wav_host_buf[2] if self._enable_c2w else None
        # each slot's own next-input row: a slot whose next_embed is this view feeds the step
        # what the previous step computed on the device; any other tensor there (the engine
        # loop's codec_sum + text, engine_loop.py:2170-2197) is copied in before the step
        self._own_next = [self.next_x[i] for i in range(S)]

    def _reset_slot_state(self, slot_id: int) -> None:
        with torch.cuda.stream(self._stream):  # ordered before the steps that read it
            self.counts[slot_id].zero_()

    def _configure_sampling(self, slot: SlotState) -> None:
        """Per-slot sampling parameters (executor.py:1212-1227, 1335-1350), written on the
        step stream so the next step sees them."""
        sid = slot.slot_id
        identity = slot.session_id if slot.session_id is not None else f"slot:{sid}"
        seed = stable_sampling_seed(self._random_seed, identity, slot.segment_idx)
        slot.sampling_seed = seed
        self._write_sampling_state(sid, seed)

    def _write_sampling_state(self, sid: int, seed: int) -> None:
        with torch.cuda.stream(self._stream):
            self.noise_key[sid] = seed
            self.noise_step[sid] = 0
            self.temperature[sid] = self._temperature if self._do_sample else 1.0
            self.penalty[sid] = self._repetition_penalty

    def _io(self, n_rows: int, n_new: int, x_in: torch.Tensor, sample: int, parity: int = 2) -> _lib.StepIO:
        io = _lib.StepIO()
        io.slots = self.slots_buf[parity].data_ptr()
        io.n_rows = n_rows
        io.n_new = n_new
        io.slot_indexed = 1
        io.x_in = x_in.data_ptr()
        io.token_counts = self.counts.data_ptr()
        if self._do_sample:
            io.noise_seed = self._random_seed & _MAX_SEED
            io.noise_key = self.noise_key.data_ptr()
            io.noise_step = self.noise_step.data_ptr()
        else:
            io.gumbel = self.zero_gumbel.data_ptr()
            io.cp_gumbel = self.zero_cp_gumbel.data_ptr()
        io.temperature = self.temperature.data_ptr()
        io.penalty = self.penalty.data_ptr()
        io.sample = sample
        io.text_add = self.text_add.data_ptr()
        io.hidden_out = self.hidden.data_ptr()
        io.logits_out = self.logits.data_ptr()
        io.full_codec_out = self.codes_buf[parity].data_ptr()
        io.codec_sum_out = self.codec_sum_buf[parity].data_ptr()
        io.next_x_out = self.next_x.data_ptr()
        io.status = self.status.data_ptr()
        return io

    def set_text_embedding(self, slot: SlotState, emb: Optional[torch.Tensor]) -> None:
        """Text embedding added to the codec sum to form the slot's next input
        (engine_loop.py:2170-2203: trailing[text_idx] or tts_pad)."""
        self._stream.wait_stream(torch.cuda.current_stream(self._device))  # emb may come from that stream
        with torch.cuda.stream(self._stream):
            if emb is None:
                self.text_add[slot.slot_id].zero_()
            else:
                self.text_add[slot.slot_id].copy_(emb.reshape(-1).to(self._device, torch.float32), non_blocking=True)

    # -- prefill ----------------------------------------------------------
    def _validate_prefill_len(self, seq: int, stage: str) -> None:
        if seq > self._max_input_len:
            raise ValueError(f"{stage} input length {seq} exceeds max_input_len={self._max_input_len}; "
                             "split the request into shorter segments")

    def _prefill_call(self, slot: SlotState, embeds: torch.Tensor, sample: int) -> None:
        seq = int(embeds.shape[-2]) if embeds.dim() == 3 else int(embeds.shape[0])
        x = embeds.reshape(seq, -1).to(self._device, torch.float32).contiguous()
        self._stream.wait_stream(torch.cuda.current_stream(self._device))  # x is made on that stream
        with torch.cuda.stream(self._stream):
            self.slots_dev[:1].fill_(slot.slot_id)
            self._model.step(self._io(1, seq, x, sample), self._stream)
            self.status_host.copy_(self.status, non_blocking=True)
        self._stream.synchronize()
        _lib.check(int(self.status_host[0]), "prefill scheduler")
        slot.past_len += seq

    def _first_frame_audio(self, slot: SlotState) -> Optional[bytes]:
        """Code2wav of the frame a prefill sampled (the fused prefill runs code2wav on it:
        executor.py:859-877), from zero decoder state — or from the warm state
        ``apply_c2w_warm_state`` installed for this session."""
        if self._c2w is None:
            return None
        warm = self._c2w_warm.pop(slot.slot_id, None)
        cs = self._c2w_stream  # every code2wav call runs on this stream, in order
        cs.wait_stream(self._stream)
        with torch.cuda.stream(cs):
            if warm is None or warm != slot.session_id:
                self._c2w.reset(self.slots_dev[:1], stream=cs)
            self._c2w.step(self.codes, self.slots_dev, self.wav, n=1, stream=cs)
            self.wav_host[:1].copy_(self.wav[:1], non_blocking=True)
        cs.synchronize()
        return self.wav_host[0].numpy().tobytes()

    def prefill(self, slot: SlotState, prefill_embeds: torch.Tensor):
        """executor.py:759-877: KV for the prompt plus the first frame's codes and audio."""
        seq = int(prefill_embeds.shape[1])
        self._validate_prefill_len(seq, "prefill")
        self._kv_pool.init_kv_tensors(slot)
        self._configure_sampling(slot)
        self._prefill_call(slot, prefill_embeds, sample=1)
        slot.position_offset = 0
        slot.frame_idx += 1
        slot.next_embed = self._own_next[slot.slot_id]
        audio = self._first_frame_audio(slot)
        codes = self.codes[:1].cpu()
        return audio, bool(int(codes[0, 0]) == self._config.talker.codec_eos_id)

    def iter_prefill(self, slot: SlotState, prefill_embeds: torch.Tensor, chunk: int = 128, keep_kv: bool = False):
        """Chunked prefill (the first "next" item after the decode step: prefill interleaved with
        decode).  A generator: each ``next()`` runs one engine step over the following
        ``chunk`` prompt tokens (KV appended after the previous chunk's; no sampling) and yields
        ``None``; the last chunk samples the first frame, and the final ``next()`` yields
        ``prefill``'s ``(audio bytes, eos)``.  A serving loop calls ``next()`` between decode
        steps, so a long prompt never stalls the running streams for more than one chunk.
        Prompts longer than ``max_prefill_rows`` are accepted (each chunk is at most that).
        ``keep_kv``: append after the KV the slot already holds (a restored or freshly cached
        prefix), as ``prefill_from_prefix`` does, instead of starting an empty sequence."""
        seq = int(prefill_embeds.shape[1])
        if chunk < 1:
            raise ValueError("chunk must be >= 1")
        chunk = min(chunk, self._max_input_len)
        if not keep_kv:
            self._kv_pool.init_kv_tensors(slot)
        self._configure_sampling(slot)
        for start in range(0, seq, chunk):
            last = start + chunk >= seq
            self._prefill_call(slot, prefill_embeds[:, start:start + chunk], sample=1 if last else 0)
            if not last:
                yield None
        slot.position_offset = 0
        slot.frame_idx += 1
        slot.next_embed = self._own_next[slot.slot_id]
        audio = self._first_frame_audio(slot)
        codes = self.codes[:1].cpu()
        yield audio, bool(int(codes[0, 0]) == self._config.talker.codec_eos_id)

    def prefill_chunked(self, slot: SlotState, prefill_embeds: torch.Tensor, chunk: int = 128):
        """``prefill`` cut into engine steps of at most ``chunk`` tokens (see ``iter_prefill``)."""
        result = None
        for result in self.iter_prefill(slot, prefill_embeds, chunk):
            pass
        return result

    def prefill_prefix_only(self, slot: SlotState, prefill_embeds: torch.Tensor) -> None:
        """executor.py:879-950: KV for a cacheable prefix, no sampling."""
        seq = int(prefill_embeds.shape[1])
        self._validate_prefill_len(seq, "prefill_prefix_only")
        self._kv_pool.init_kv_tensors(slot)
        self._prefill_call(slot, prefill_embeds, sample=0)
        slot.position_offset = 0

    def prefill_from_prefix(self, slot: SlotState, request_prefill_embeds: torch.Tensor):
        """executor.py:952-1081: append a suffix on top of the slot's (shared) KV."""
        seq = int(request_prefill_embeds.shape[1])
        self._validate_prefill_len(seq, "prefill_from_prefix")
        self._configure_sampling(slot)
        self._prefill_call(slot, request_prefill_embeds, sample=1)
        slot.frame_idx += 1
        slot.next_embed = self._own_next[slot.slot_id]
        audio = self._first_frame_audio(slot)
        codes = self.codes[:1].cpu()
        return audio, bool(int(codes[0, 0]) == self._config.talker.codec_eos_id)

    # -- decode -----------------------------------------------------------
    def _step_a(self, io: _lib.StepIO) -> None:
        """Talker + sampling + code predictor + codec sum (stream A)."""
        self._model.step(io, self._stream)

    def _step_b(self, n: int, parity: int) -> None:
        """Code2wav of the step's frame (stream B)."""
        self._c2w.step(self.codes_buf[parity], self.slots_buf[parity], self.wav, n=n, stream=self._c2w_stream)

    def _capture(self, n: int):
        """CUDA graphs of both parities: (graph A, graph B or None) per parity, and the launch count."""
        graphs = []
        launches = 0
        for par in (0, 1):
            io = self._io(n, 1, self.next_x, sample=1, parity=par)
            ga = torch.cuda.CUDAGraph()
            with torch.cuda.graph(ga, stream=self._stream):
                self._step_a(io)
            gb = None
            if self._c2w is not None:
                gb = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gb, stream=self._c2w_stream):
                    self._step_b(n, par)
                io.launches += self._c2w.last_launches
            graphs.append((ga, gb))
            launches = io.launches
        return graphs, launches

    def _enqueue_step(self, n: int, upload: bool, graphs=None):
        """Enqueue one decode step of the first n slots of the next parity's slot buffer.
        Returns (parity, event after stream A's part, event after the whole step)."""
        par = self._parity
        self._parity ^= 1
        a, b = self._stream, self._c2w_stream
        with torch.cuda.stream(a):
            if self._done_b[par] is not None:  # code2wav of step t - 2 has read this parity's buffers
                a.wait_event(self._done_b[par])
            if upload:
                self.slots_buf[par][:n].copy_(self.slots_host_buf[par][:n], non_blocking=True)
            if graphs is not None:
                graphs[par][0].replay()
            else:
                self._step_a(self._io(n, 1, self.next_x, sample=1, parity=par))
            self.codes_host_buf[par][:n].copy_(self.codes_buf[par][:n], non_blocking=True)
            self.status_host_buf[par].copy_(self.status, non_blocking=True)
            ev_a = torch.cuda.Event()
            ev_a.record(a)
        ev_b = ev_a
        if self._c2w is not None:
            b.wait_event(ev_a)
            with torch.cuda.stream(b):
                if graphs is not None:
                    graphs[par][1].replay()
                else:
                    self._step_b(n, par)
                self.wav_host_buf[par][:n].copy_(self.wav[:n], non_blocking=True)
                ev_b = torch.cuda.Event()
                ev_b.record(b)
        self._done_a[par] = ev_a
        self._done_b[par] = ev_b
        return par, ev_a, ev_b

    def prepare_replay(self, slots: List[SlotState]):
        """Upload `slots` to both parities' slot buffers and capture the batch's graphs (for
        timing loops that replay the same batch); returns the launches per step."""
        n = len(slots)
        for par in (0, 1):
            self.slots_host_buf[par][:n].numpy()[:] = [s.slot_id for s in slots]
            self.slots_buf[par][:n].copy_(self.slots_host_buf[par][:n])
        torch.cuda.synchronize(self._device)
        g = self._graphs.get(n)
        if g is None:
            g = self._capture(n)
            self._graphs[n] = g
        return g[1]

    def capture_graphs(self, sizes) -> None:
        """Capture the decode-step CUDA graphs of every batch size in ``sizes`` ahead of time (a
        serving loop whose batch size changes every few steps would otherwise pay a capture the
        second time each size occurs)."""
        torch.cuda.synchronize(self._device)
        for n in sizes:
            n = int(n)
            if not 1 <= n <= self._max_batch:
                raise ValueError(f"batch size {n} outside [1, {self._max_batch}]")
            if self._graphs.get(n) is None:
                self._graphs[n] = self._capture(n)
        torch.cuda.synchronize(self._device)

    def replay_step(self, n: int):
        """One decode step of the batch `prepare_replay` set up; returns (event after
        stream A's part, event after the whole step).  The host does not wait."""
        _, ev_a, ev_b = self._enqueue_step(n, upload=False, graphs=self._graphs[n][0])
        return ev_a, ev_b

    def launch_decode_step(self, slots: List[SlotState]) -> GPUFuture:
        """executor.py:1087-1183 — enqueue one decode step and return at once."""
        n = len(slots)
        if n == 0 or n > self._max_batch:
            raise ValueError(f"batch of {n} slots outside [1, {self._max_batch}]")
        if len({s.slot_id for s in slots}) != n:
            # two rows of one slot would append to the same block-table row and KV position
            raise ValueError("a decode batch lists the same slot twice")
        cap = self._max_seq_len
        for s in slots:
            if s.past_len + 1 > cap:
                raise ValueError(f"slot {s.slot_id} is at max_seq_len={cap}")
        original = [s.past_len for s in slots]
        self._kv_pool.flush_drops()
        self._stage_host_inputs(slots)
        par = self._parity
        if self._done_a[par] is not None:  # the staging copy of step t - 2 has been consumed
            self._done_a[par].synchronize()
        self.slots_host_buf[par][:n].numpy()[:] = [s.slot_id for s in slots]
        graphs = None
        if self._use_graphs:
            if n not in self._graphs:
                self._graphs[n] = None  # first step of this batch size runs eagerly
            elif self._graphs[n] is None:
                torch.cuda.synchronize(self._device)
                self._graphs[n] = self._capture(n)
            if self._graphs[n] is not None:
                graphs = self._graphs[n][0]
        par, ev_a, ev_b = self._enqueue_step(n, upload=True, graphs=graphs)
        own = self._own_next
        for s in slots:  # the device formed each slot's next input; the loop may replace it
            s.next_embed = own[s.slot_id]
        return GPUFuture(_executor=self, _event=ev_b, _slots=list(slots), _original_past_lens=original,
                         _codes_host=self.codes_host_buf[par], _codes_dev=self.codes_buf[par],
                         _codec_sum=BatchRows(self.codec_sum_buf[par], [s.slot_id for s in slots]),
                         _status_host=self.status_host_buf[par],
                         _wav_host=self.wav_host_buf[par] if self._c2w is not None else None)

    @staticmethod
    def advance(slots: List[SlotState]) -> None:
        """The per-slot counters the engine loop advances for each decode step it launched
        (engine_loop.py:2163-2165): a caller that drives ``launch_decode_step`` without the
        reference loop calls this once per launched step, before launching the next one."""
        for s in slots:
            s.past_len += 1
            s.frame_idx += 1
            s.touch()

    def _stage_host_inputs(self, slots: List[SlotState]) -> None:
        """What the reference engine loop hands a decode step through its slots.

        * A slot whose ``next_embed`` is not the device's own row (the loop sets
          ``codec_sum + trailing text`` itself, engine_loop.py:2170-2197, or a primed prefix
          suffix, 913-928) has that tensor copied into its input row before the step.
        * A slot at ``frame_idx == 0`` starts a stream without a prefill of this executor (a
          prefix-cache hit or a prefix-only prefill primed by the loop, engine_loop.py:801-835,
          893-928): its sampling state is set and its code2wav state zeroed, as ``prefill``
          does for the streams it starts.
        """
        own = self._own_next
        moved = [s for s in slots if s.next_embed is not None and s.next_embed is not own[s.slot_id]]
        fresh = [s for s in slots if s.frame_idx == 0]
        if not moved and not fresh:
            return
        for s in fresh:
            self._configure_sampling(s)
        self._apply_host_inputs(moved, fresh)

    def _apply_host_inputs(self, moved: List[SlotState], fresh: List[SlotState]) -> None:
        """Device side of ``_stage_host_inputs``: copy the moved inputs in, zero the fresh
        streams' code2wav state."""
        cur = torch.cuda.current_stream(self._device)
        self._stream.wait_stream(cur)  # the loop made its tensors on that stream
        with torch.cuda.stream(self._stream):
            if moved:
                for s in moved:
                    if s.next_embed.is_cuda:
                        s.next_embed.record_stream(self._stream)
                rows = torch.cat([s.next_embed.reshape(1, -1).to(self._device, torch.float32) for s in moved])
                idx = torch.tensor([s.slot_id for s in moved], dtype=torch.long, device=self._device)
                self.next_x.index_copy_(0, idx, rows)
        if fresh and self._c2w is not None:
            b = self._c2w_stream
            b.wait_stream(self._stream)
            with torch.cuda.stream(b):
                ids = torch.tensor([s.slot_id for s in fresh], dtype=torch.int32, device=self._device)
                self._c2w.reset(ids, stream=b)

    def warmup(self, n_rounds: int = 3) -> None:
        """executor.py:1541-1605: a throw-away slot through prefill and decode."""
        slot = self._kv_pool.allocate("__warmup__")
        if slot is None:
            return
        try:
            dummy = torch.randn(1, 4, self._config.talker.hidden_size, device=self._device) * 0.02
            self.prefill(slot, dummy)
            for _ in range(n_rounds):
                self.launch_decode_step([slot]).wait()
                self.advance([slot])
        finally:
            self._kv_pool.release(slot.slot_id)
