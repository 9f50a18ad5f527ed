"""Host-side engine logic on CPU: block manager (against the reference's own
allocation traces), scheduler pressure paths, request lifecycle, prompt layout,
checkpoint writer / loader, and bucket selection. No GPU needed."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.conftest import load_json
from voiceagent_b200.audio.frontend import AudioFeatures
from voiceagent_b200.config import EngineConfig
from voiceagent_b200.engine.block_manager import BlockManager
from voiceagent_b200.engine.request import AsrRequest, RequestStage, SamplingParams
from voiceagent_b200.engine.scheduler import ModelBatch, Scheduler
from voiceagent_b200.prompt import PromptBuilder, PromptLayout, normalize_language

BS = 256
AUDIO = 151676


def make_request(prompt_len, audio_offset=8, audio_length=13, max_new_tokens=440):
    suffix = prompt_len - audio_offset - audio_length
    ids = (list(range(1000, 1000 + audio_offset)) + [AUDIO] * audio_length
           + list(range(2000, 2000 + suffix)))
    frames = max(1, audio_length * 100 // 13)
    return AsrRequest(
        features=AudioFeatures(mel=torch.zeros(128, frames), mel_frames=frames,
                               num_audio_tokens=audio_length, audio_seconds=audio_length / 13),
        layout=PromptLayout(token_ids=ids, audio_offset=audio_offset, audio_length=audio_length),
        sampling=SamplingParams(max_new_tokens=max_new_tokens), block_size=BS,
        stop_token_ids={151643, 151645})


@pytest.fixture
def config(tmp_path):
    from voiceagent_b200.checkpoint import write_checkpoint

    path = write_checkpoint(tmp_path / "ckpt", "tiny", weights=False)

    def build(**kw):
        settings = dict(model=str(path), max_num_seqs=8, max_model_len=4096,
                        max_num_batched_tokens=4096)
        settings.update(kw)
        return EngineConfig(**settings)

    return build


def admit_for_prefill(scheduler, request):
    request.audio_embeds = torch.zeros(request.layout.audio_length, 4)
    request.stage = RequestStage.WAITING_PREFILL
    scheduler.admit_prefill([request])
    return request


def start_decoding(scheduler, manager, request):
    admit_for_prefill(scheduler, request)
    manager.allocate(request)
    request.num_computed_tokens = len(request)
    request.stage = RequestStage.RUNNING_DECODE
    scheduler.waiting_prefill.remove(request)
    scheduler.running.append(request)
    return request


# ------------------------------------------------------------- block manager


@pytest.mark.parametrize("trace_index", [0, 1])
def test_block_manager_reproduces_reference_traces(trace_index):
    trace = load_json("block_manager.json")[trace_index]
    manager = BlockManager(num_blocks=24, block_size=BS, enable_prefix_cache=trace["prefix_cache"])
    reqs = {}
    for entry in trace["log"]:
        if entry["op"] == "alloc":
            r = make_request(*entry["arg"])
            reqs[entry["name"]] = r
            ok = manager.can_allocate(r)
            assert ok == entry["ok"]
            if ok:
                manager.allocate(r)
            assert r.block_table == entry["table"]
            assert (r.num_cached_tokens, r.num_computed_tokens) == (entry["cached"], entry["computed"])
        elif entry["op"] == "append":
            r = reqs[entry["name"]]
            for step in range(entry["arg"]):
                r.append_token(5000 + step)
                if manager.can_append(r):
                    manager.may_append(r)
            assert r.block_table == entry["table"]
        else:
            manager.deallocate(reqs[entry["name"]])
            assert list(manager.free_block_ids) == entry["free_order"]
        assert manager.num_free_blocks == entry["free"]
    assert BlockManager.compute_hash(list(range(256))) == trace["hash_example"]


def test_prefix_reuse_and_audio_isolation():
    manager = BlockManager(num_blocks=32, block_size=BS)
    first = make_request(700, 609, 46)
    second = make_request(700, 609, 46)
    manager.allocate(first)
    manager.allocate(second)
    assert second.num_cached_tokens == 2 * BS
    assert second.block_table[:2] == first.block_table[:2]
    assert second.block_table[2] != first.block_table[2]
    a, b = make_request(600, 0, 590), make_request(600, 0, 590)
    manager.allocate(a)
    manager.allocate(b)
    assert b.num_cached_tokens == 0 and set(a.block_table).isdisjoint(b.block_table)


def test_append_allocates_only_on_block_boundary():
    manager = BlockManager(num_blocks=8, block_size=BS)
    r = make_request(BS, 9, 46)
    manager.allocate(r)
    r.append_token(42)
    assert manager.can_append(r)
    manager.may_append(r)
    assert len(r.block_table) == 2
    r.append_token(43)
    manager.may_append(r)
    assert len(r.block_table) == 2


# ----------------------------------------------------------------- scheduler


def test_preempts_newest_to_keep_oldest(config):
    manager = BlockManager(2, BS)
    s = Scheduler(config(), manager)
    first = start_decoding(s, manager, make_request(BS))
    second = start_decoding(s, manager, make_request(BS))
    first.append_token(7)
    second.append_token(7)
    batch = s.schedule_model()
    assert batch.decode == [first]
    assert s.stats.num_preemptions == 1
    assert second.stage is RequestStage.WAITING_PREFILL and second.block_table == []
    assert second.audio_embeds is not None and second.num_computed_tokens == 0


def test_lone_request_that_cannot_grow_is_aborted(config):
    manager = BlockManager(1, BS)
    s = Scheduler(config(), manager)
    only = start_decoding(s, manager, make_request(BS))
    only.append_token(7)
    assert not s.schedule_model()
    assert s.drain_aborted() == [only]
    assert only.finish_reason == "aborted:out_of_kv_blocks" and not s.has_work


def test_unplaceable_request_is_aborted_not_stalled(config):
    s = Scheduler(config(), BlockManager(2, BS))
    r = admit_for_prefill(s, make_request(3 * BS))
    assert not s.schedule_model()
    assert s.drain_aborted() == [r] and r.finish_reason == "aborted:kv_cache_too_small"


def test_transient_pressure_waits(config):
    manager = BlockManager(2, BS)
    s = Scheduler(config(), manager)
    start_decoding(s, manager, make_request(BS))
    blocked = admit_for_prefill(s, make_request(2 * BS))
    s.schedule_model()
    assert not s.aborted and list(s.waiting_prefill) == [blocked]


def test_model_oom_rollback_and_cap(config):
    manager = BlockManager(32, BS)
    s = Scheduler(config(max_num_seqs=8), manager)
    reqs = [admit_for_prefill(s, make_request(BS)) for _ in range(8)]
    batch = s.schedule_model()
    assert len(batch.prefill) == 8
    s.on_model_oom(batch)
    assert list(s.waiting_prefill) == reqs
    assert all(r.block_table == [] and r.num_computed_tokens == 0 for r in reqs)
    assert s.model_batch_limit == 4
    assert len(s.schedule_model().requests) == 4
    s.relax_limits()
    assert s.model_batch_limit == 8


def test_single_request_oom_gives_up(config):
    manager = BlockManager(16, BS)
    s = Scheduler(config(), manager)
    r = start_decoding(s, manager, make_request(BS // 2))
    s.on_model_oom(s.schedule_model())
    assert s.drain_aborted() == [r] and r.finish_reason == "aborted:out_of_memory"


def test_audio_oom_requeues_in_order(config):
    s = Scheduler(config(max_audio_batch_frames=10_000), BlockManager(16, BS))
    reqs = [make_request(BS) for _ in range(3)]
    for r in reqs:
        s.add(r)
    picked = s.schedule_audio()
    assert picked == reqs
    s.on_audio_oom(picked)
    assert list(s.waiting_encode) == reqs and s.audio_frame_limit < 10_000


def test_postprocess_finishes_and_frees(config):
    manager = BlockManager(8, BS)
    s = Scheduler(config(), manager)
    r = make_request(60, 9, 46, max_new_tokens=2)
    admit_for_prefill(s, r)
    batch = s.schedule_model()
    assert batch.prefill == [r] and r.num_tokens_to_compute == 60
    assert s.postprocess(batch, [11]) == []
    assert r.stage is RequestStage.RUNNING_DECODE and r.num_tokens_to_compute == 1
    batch = s.schedule_model()
    assert batch.decode == [r]
    assert s.postprocess(batch, [12]) == [r]
    assert r.finish_reason == "length" and manager.num_free_blocks == 8


def test_cancel_waiting_request(config):
    s = Scheduler(config(), BlockManager(8, BS))
    r = make_request(60, 9, 46)
    s.add(r)
    assert s.cancel(r.request_id)
    assert s.drain_aborted() == [r] and r.finish_reason == "cancelled"
    assert not s.cancel(12345678)


def test_empty_batch_rollback_is_noop(config):
    s = Scheduler(config(), BlockManager(16, BS))
    s.on_model_oom(ModelBatch())
    assert not s.aborted and not s.has_work


# ---------------------------------------------------------- request / prompt


def test_request_lifecycle():
    r = make_request(62, 9, 46)
    assert r.num_tokens_to_compute == 62
    r.num_computed_tokens = 62
    r.append_token(7)
    assert r.num_tokens_to_compute == 1
    r.append_token(151645)
    assert r.check_finished() and r.finish_reason == "stop"


def test_sampling_for_audio():
    assert SamplingParams().max_new_tokens == 440
    assert SamplingParams.for_audio(5.0).max_new_tokens == 440
    assert SamplingParams.for_audio(1299.0).max_new_tokens > 4849
    assert SamplingParams.for_audio(1200.0, max_new_tokens=99).max_new_tokens == 99


def test_prompt_template_ids():
    # pinned by the reference's tests/test_prompt.py:24-47
    layout = PromptBuilder().build(1)
    assert layout.token_ids == [151644, 8948, 198, 151645, 198, 151644, 872, 198, 151669, 151676,
                                151670, 151645, 198, 151644, 77091, 198]
    assert layout.audio_offset == 9
    forced = PromptBuilder().build(46, language="English")
    assert forced.token_ids[-1] == 151704 and len(forced) == 46 + 18
    assert forced.token_ids[9:55] == [151676] * 46
    with pytest.raises(ValueError):
        PromptBuilder().build(0)
    assert normalize_language("EN") == "English" and normalize_language("") is None


# ------------------------------------------------------ checkpoint / loader


def test_engine_and_oracle_random_init_agree():
    from oracle import model as M
    from voiceagent_b200.checkpoint import PRESETS, random_state_dict

    cfg = PRESETS["tiny"]
    ours = random_state_dict(cfg, seed=3, dtype=torch.float32)
    theirs = M.init_weights(cfg, seed=3)
    assert set(ours) == set(theirs) - ({"lm_head.weight"} if "lm_head.weight" not in ours else set())
    for name, t in ours.items():
        assert torch.equal(t, theirs[name]), name


def test_checkpoint_roundtrip_into_fused_model(tmp_path):
    from voiceagent_b200.checkpoint import random_state_dict, write_checkpoint
    from voiceagent_b200.config import Qwen3ASRConfig
    from voiceagent_b200.loader import load_weights
    from voiceagent_b200.qwen3_asr.model import Qwen3ASRForConditionalGeneration

    path = write_checkpoint(tmp_path / "c", "tiny", seed=5)
    cfg = Qwen3ASRConfig.from_pretrained(str(path))
    assert cfg.stop_token_ids == [151643, 151645] and cfg.text.hidden_size == 256
    torch.set_default_dtype(torch.bfloat16)
    try:
        model = Qwen3ASRForConditionalGeneration(cfg, 4096)
    finally:
        torch.set_default_dtype(torch.float32)
    load_weights(model, str(path))
    ref = random_state_dict("tiny", seed=5)
    qkv = model.model.layers[1].self_attn.qkv_proj.weight
    assert torch.equal(qkv[:512], ref["model.layers.1.self_attn.q_proj.weight"])
    assert torch.equal(qkv[512:768], ref["model.layers.1.self_attn.k_proj.weight"])
    enc = model.audio_tower.layers[0].self_attn.qkv_proj.bias
    assert torch.equal(enc[128:256], ref["audio_tower.layers.0.self_attn.k_proj.bias"])
    assert model.lm_head.weight is model.model.embed_tokens.weight


def test_loader_rejects_orphans(tmp_path):
    from safetensors.torch import save_file

    from voiceagent_b200.checkpoint import random_state_dict, write_checkpoint
    from voiceagent_b200.config import Qwen3ASRConfig
    from voiceagent_b200.loader import load_weights
    from voiceagent_b200.qwen3_asr.model import Qwen3ASRForConditionalGeneration

    path = write_checkpoint(tmp_path / "c", "tiny", weights=False)
    tensors = {"thinker." + k: v for k, v in random_state_dict("tiny").items()}
    tensors["thinker.bogus.weight"] = torch.zeros(1)
    save_file(tensors, str(path / "model.safetensors"))
    model = Qwen3ASRForConditionalGeneration(Qwen3ASRConfig.from_pretrained(str(path)), 4096)
    with pytest.raises(RuntimeError, match="no destination"):
        load_weights(model, str(path))


def test_bucket_selection():
    from voiceagent_b200.engine.graph_runner import DEFAULT_BUCKETS, GraphRunner

    runner = GraphRunner.__new__(GraphRunner)
    runner.buckets = DEFAULT_BUCKETS
    assert [runner.bucket_for(n) for n in (1, 3, 16, 17, 64)] == [1, 4, 16, 24, 64]
    assert runner.bucket_for(65) is None


def test_audio_token_accounting_matches_oracle():
    from oracle import kernels as K
    from voiceagent_b200.audio import tokens as T

    for f in range(1, 3000):
        assert T.num_audio_tokens(f) == K.num_audio_tokens(f)
        assert T.chunk_lengths_for(f) == K.chunk_lengths_for(f)
    assert T.attention_window_tokens(800) == 104


# ------------------------------------------------------------ multi-step decode


def test_may_append_matches_reference_rule_and_is_idempotent():
    manager = BlockManager(64, BS, enable_prefix_cache=False)
    r = make_request(BS - 1)
    manager.allocate(r)
    for _ in range(3 * BS):
        held = len(r.block_table)
        r.append_token(7)
        manager.may_append(r)
        assert len(r.block_table) - held == (1 if len(r) % BS == 1 else 0)  # reference rule
        manager.may_append(r)  # again: nothing more
        assert len(r.block_table) == r.num_blocks


def test_lookahead_blocks_cover_every_written_position():
    manager = BlockManager(64, BS, enable_prefix_cache=False)
    r = make_request(BS - 2)
    manager.allocate(r)
    for steps in (1, 2, 3, 4):
        need = manager.blocks_ahead(r, steps)
        assert need == max(0, -(-(len(r) + steps - 1) // BS) - len(r.block_table))
    manager.append_ahead(r, 4)  # positions len-1 .. len+2 cross into the next block
    assert len(r.block_table) * BS >= len(r) + 3
    assert manager.blocks_ahead(r, 4) == 0


def test_decode_steps_bounded_by_budget_length_blocks_and_cancel(config):
    manager = BlockManager(64, BS)
    scheduler = Scheduler(config(), manager)
    a, b = make_request(60, max_new_tokens=10), make_request(70, max_new_tokens=3)
    for r in (a, b):
        start_decoding(scheduler, manager, r)
    batch = scheduler.schedule_model()
    assert batch.decode == [a, b]
    assert scheduler.decode_steps_for(batch, 4, max_model_len=4096) == 3  # b: 3 tokens of budget
    assert scheduler.decode_steps_for(batch, 4, max_model_len=len(a)) == 1  # model length
    assert scheduler.decode_steps_for(batch, 1, max_model_len=4096) == 1
    b.cancel_requested = True
    assert scheduler.decode_steps_for(batch, 4, max_model_len=4096) == 1


def test_multi_step_postprocess_equals_single_steps(config):
    def run(multi):
        manager = BlockManager(64, BS)
        scheduler = Scheduler(config(), manager)
        reqs = [make_request(BS - 2 + i, max_new_tokens=6) for i in range(3)]
        for r in reqs:
            start_decoding(scheduler, manager, r)
        rng = np.random.default_rng(5)
        tokens = [[int(t) for t in rng.integers(100, 200, size=3)] for _ in range(3)]
        tokens[1][2] = 151645  # request 2 stops on EOS at the second step
        batch = scheduler.schedule_model()
        finished = []
        if multi:
            assert scheduler.decode_steps_for(batch, 3, max_model_len=4096) == 3
            finished += scheduler.postprocess_steps(batch, tokens)
        else:
            for k in range(3):
                step = [tokens[k][reqs.index(r)] for r in batch.decode]
                finished += scheduler.postprocess(batch, step)
                batch = scheduler.schedule_model()
        state = [(list(r.token_ids), r.stage, len(r.block_table)) for r in reqs]
        return state, [r.request_id - reqs[0].request_id for r in finished], manager.num_free_blocks
    single, multi = run(False), run(True)
    assert single == multi
    assert multi[1] == [2]  # the EOS request finished; its third token was discarded


def test_batched_record_equals_per_token_record(config):
    """Scheduler._record_run (one append per request and call) leaves every request as
    the per-token _record loop does: tokens kept, computed count, stage, finish reason;
    over stop tokens at every position, caps reached before, at and after the stop,
    ignore_eos and cancels."""
    scheduler = Scheduler(config(), BlockManager(64, BS))
    rng = np.random.default_rng(11)
    stop = 151645
    for case in range(2000):
        steps = int(rng.integers(1, 5))
        run = tuple(int(t) for t in rng.integers(100, 200, size=steps))
        if rng.random() < 0.6:
            run = tuple(stop if rng.random() < 0.3 else t for t in run)
        made = []
        for _ in range(2):
            r = make_request(40, max_new_tokens=int(rng.integers(1, 8)))
            r.stage = RequestStage.RUNNING_DECODE
            made.append(r)
        outputs = int(rng.integers(0, 9))
        ignore, cancel = rng.random() < 0.2, rng.random() < 0.05
        for r in made:
            r.token_ids += [150] * outputs
            r.num_computed_tokens = len(r) - 1
            r.sampling.max_new_tokens = made[0].sampling.max_new_tokens
            r.sampling.ignore_eos, r.cancel_requested = ignore, cancel
        per_token = any(scheduler._record(made[0], t) for t in run)
        batched = scheduler._record_run(made[1], run)
        want, got = made
        assert (per_token, want.token_ids, want.num_computed_tokens, want.stage, want.finish_reason) \
            == (batched, got.token_ids, got.num_computed_tokens, got.stage, got.finish_reason), \
            (case, run, outputs, want.sampling)


def test_waveform_staging_during_decode_respects_queue_order_cap_and_budget():
    """AsrEngine._stage_upcoming_audio (run while a decoder call executes) stages the
    head of the encode queue in order, at most one encoder call's worth, skips clips
    already staged, and stops after the first clip past its time budget."""
    from collections import deque
    from types import SimpleNamespace

    from voiceagent_b200.engine.engine import AsrEngine

    staged = []

    def stage(features):
        if features in staged:
            return False
        staged.append(features)
        return True

    queue = deque(SimpleNamespace(features=f"clip{i}") for i in range(10))
    fake = SimpleNamespace(scheduler=SimpleNamespace(waiting_encode=queue),
                           config=SimpleNamespace(max_audio_batch_size=4),
                           audio_runner=SimpleNamespace(renderer=SimpleNamespace(stage=stage)))
    AsrEngine._stage_upcoming_audio(fake, 0.0)  # no budget: one clip per call
    assert staged == ["clip0"]
    AsrEngine._stage_upcoming_audio(fake, 0.0)
    assert staged == ["clip0", "clip1"]
    AsrEngine._stage_upcoming_audio(fake, 10.0)  # the rest of the next encoder call
    assert staged == ["clip0", "clip1", "clip2", "clip3"]
    queue.popleft()
    AsrEngine._stage_upcoming_audio(fake, 10.0)
    assert staged[-1] == "clip4" and len(staged) == 5


def _reference_take_decodes(scheduler, batch):
    """The per-request form of Scheduler._take_decodes (the reference's loop)."""
    bm = scheduler.block_manager
    while scheduler.running:
        if bm.can_append(scheduler.running[0]):
            batch.decode.append(scheduler.running.popleft())
        elif len(scheduler.running) > 1:
            scheduler._preempt(scheduler.running.pop())
        else:
            scheduler._retire(scheduler.running.popleft(), "aborted:out_of_kv_blocks")
            return


def _reference_decode_steps_for(scheduler, batch, limit, max_model_len):
    """The per-request form of Scheduler.decode_steps_for."""
    if limit <= 1 or batch.prefill or not batch.decode:
        return 1
    if any(r.cancel_requested for r in batch.decode):
        return 1
    steps = min([limit] + [min(r.sampling.max_new_tokens - r.num_output_tokens,
                               max_model_len - len(r) + 1) for r in batch.decode])
    if steps <= 1:
        return 1
    bm = scheduler.block_manager
    if sum(bm.blocks_ahead(r, steps) for r in batch.decode) > bm.num_free_blocks:
        return 1
    for r in batch.decode:
        bm.append_ahead(r, steps)
    return steps


def _random_decode_state(config, rng, n_blocks):
    manager = BlockManager(n_blocks, BS, enable_prefix_cache=False)
    scheduler = Scheduler(config(max_num_seqs=16), manager)
    made = []
    for _ in range(int(rng.integers(1, 7))):
        prompt = int(rng.integers(22, 3 * BS))
        outputs = int(rng.integers(0, 12))
        if rng.random() < 0.6:  # land near a block boundary: lengths BS k - 2 .. BS k + 2
            target = BS * (prompt // BS + 1) + int(rng.integers(-2, 3))
            outputs = max(0, target - prompt)
        r = make_request(prompt, max_new_tokens=outputs + int(rng.integers(2, 40)))
        if manager.num_free_blocks < -(-(prompt + outputs) // BS):  # prompt + outputs' blocks
            break
        start_decoding(scheduler, manager, r)
        r.token_ids += [150] * outputs  # outputs already sampled
        manager.may_append(r)
        made.append(r)
    # use up free blocks so that block-opening requests meet a full cache
    while manager.num_free_blocks > int(rng.integers(0, 3)):
        manager._take_any()
    return scheduler, manager, made


def test_take_decodes_equals_the_per_request_loop(config):
    """Scheduler._take_decodes' shortcut (every request joins when a block is free or none
    opens one) decides exactly as the reference's request-by-request loop: same decode
    batch, preemptions, aborts and block-manager state, over random caches near full."""
    import copy

    rng = np.random.default_rng(21)
    for case in range(300):
        scheduler, manager, made = _random_decode_state(config, rng, int(rng.integers(3, 12)))
        if not made:
            continue
        other = copy.deepcopy((scheduler, made))
        fast_batch, ref_batch = ModelBatch(), ModelBatch()
        scheduler._take_decodes(fast_batch)
        _reference_take_decodes(other[0], ref_batch)
        ids = lambda rs: [r.request_id for r in rs]
        assert ids(fast_batch.decode) == ids(ref_batch.decode), case
        assert ids(scheduler.running) == ids(other[0].running), case
        assert ids(scheduler.waiting_prefill) == ids(other[0].waiting_prefill), case
        assert ids(scheduler.aborted) == ids(other[0].aborted), case
        assert manager.num_free_blocks == other[0].block_manager.num_free_blocks, case
        assert [r.block_table for r in made] == [r.block_table for r in other[1]], case


def test_decode_steps_for_equals_the_per_request_form(config):
    """Scheduler.decode_steps_for (lengths measured once, only block-opening requests
    visited) returns the same step count and takes the same blocks as the per-request
    form, over random budgets, model lengths and nearly full caches."""
    import copy

    rng = np.random.default_rng(22)
    for case in range(300):
        scheduler, manager, made = _random_decode_state(config, rng, int(rng.integers(4, 14)))
        if not made:
            continue
        batch = scheduler.schedule_model()
        if not batch.decode or batch.prefill:
            continue
        if rng.random() < 0.05:
            batch.decode[0].cancel_requested = True
        limit = int(rng.integers(1, 6))
        max_len = int(rng.integers(BS, 4 * BS))
        other_sched, other_batch = copy.deepcopy((scheduler, batch))
        got = scheduler.decode_steps_for(batch, limit, max_len)
        want = _reference_decode_steps_for(other_sched, other_batch, limit, max_len)
        assert got == want, (case, got, want)
        assert [r.block_table for r in batch.decode] == [r.block_table for r in other_batch.decode]
        assert manager.num_free_blocks == other_sched.block_manager.num_free_blocks


def test_decode_descriptor_fill_equals_the_per_request_layout():
    """graph_runner.fill_decode_descriptor (one slice store per field) writes the same
    descriptor as a request-by-request fill: lengths, last ids, table offsets and lengths,
    the concatenated tables; untouched padding slots keep their values."""
    from types import SimpleNamespace

    from voiceagent_b200.engine.graph_runner import fill_decode_descriptor

    rng = np.random.default_rng(23)
    for case in range(200):
        m = int(rng.choice([1, 4, 8, 32, 64]))
        n = int(rng.integers(1, m + 1))
        reqs = [SimpleNamespace(token_ids=list(rng.integers(0, 1000, size=int(rng.integers(1, 600)))),
                                block_table=list(rng.integers(0, 4096, size=int(rng.integers(0, 5)))))
                for _ in range(n)]
        got = np.full(4 * m + 5 * m, -7, np.int32)
        want = got.copy()
        cursor, longest = fill_decode_descriptor(got, m, reqs)
        at = 4 * m
        for i, r in enumerate(reqs):  # the request-by-request form
            want[i] = len(r.token_ids)
            want[m + i] = r.token_ids[-1]
            want[2 * m + i] = at - 4 * m
            want[3 * m + i] = len(r.block_table)
            want[at:at + len(r.block_table)] = r.block_table
            at += len(r.block_table)
        assert cursor == at and longest == max(len(r.token_ids) for r in reqs)
        np.testing.assert_array_equal(got, want, err_msg=str(case))


def test_encoder_positions_equal_the_oracle_table():
    """The encoder's sinusoid position table (the pos operand of audio_gather_pos) equals
    the oracle's restatement of SinusoidsPositionEmbedding, in fp32 and after the bf16
    cast the encoder applies."""
    from oracle.model import sinusoid_table as oracle_table
    from voiceagent_b200.qwen3_asr.audio_encoder import sinusoid_table

    for length, channels in ((1500, 896), (1500, 1280), (13, 64)):
        got, want = sinusoid_table(length, channels), oracle_table(length, channels)
        assert got.dtype == want.dtype == torch.float32
        assert torch.equal(got, want) and torch.equal(got.bfloat16(), want.bfloat16())
