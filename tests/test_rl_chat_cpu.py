"""S-GRPO masks, rule rewards, the reflection head and chat sessions (CPU)."""
import pytest
import torch

from mamformer_b200 import MamformerConfig, MamformerForCausalLM
from mamformer_b200.chat import ChatSession, SIMPLE_CHAT_TEMPLATE, create_chat
from mamformer_b200.reflection import ReflectionModule, SelfReflectiveGenerator, add_reflection_to_model
from mamformer_b200.rewards import (RewardCalculator, code_reward, extract_boxed, format_reward, length_penalty,
                                    math_reward, parse_number, thinking_quality_reward)
from mamformer_b200.sgrpo import StochasticGRPOConfig, batch_token_masks, sample_token_mask
from mamformer_b200.tokenizer import MamformerTokenizer


def test_sgrpo_mask_rules():
    assert sample_token_mask(10, StochasticGRPOConfig(enabled=False)).all()
    cfg = StochasticGRPOConfig(enabled=True, p=0.5, alpha=3, k=6, seed=0)
    for _ in range(20):
        m = sample_token_mask(200, cfg)
        assert m[:3].all() and int(m.sum()) <= 6
    a = sample_token_mask(100, StochasticGRPOConfig(enabled=True, p=0.4, seed=7))
    b = sample_token_mask(100, StochasticGRPOConfig(enabled=True, p=0.4, seed=7))
    assert torch.equal(a, b) and 20 < int(a.sum()) < 60
    with pytest.raises(ValueError):
        StochasticGRPOConfig(enabled=True, p=0.0).validate()
    bm = batch_token_masks([5, 8], StochasticGRPOConfig(enabled=True, p=1.0), 10)
    assert bm.sum(1).tolist() == [5, 8]


def test_math_and_format_rewards():
    assert extract_boxed(r"a \boxed{\frac{1}{2}} b \boxed{7}") == [r"\frac{1}{2}", "7"]
    assert parse_number("3/4") == 0.75 and parse_number("1,000") == 1000.0 and parse_number("2e3") == 2000.0
    assert math_reward(r"<think>x</think><answer>\boxed{42}</answer>", "42") == 1.0
    assert math_reward(r"<think>x</think><answer>\boxed{41}</answer>", "42") == 0.3
    assert math_reward(r"\boxed{41}", "42") == 0.0
    assert math_reward("no box", "42") == 0.0
    assert math_reward(r"\boxed{ABC}", "abc") == 1.0
    assert format_reward("<think>a</think><answer>b</answer>") == 1.0
    assert format_reward("<answer>b</answer><think>a</think>") == 0.7
    assert format_reward("<think>a</think>") == 0.5
    assert format_reward("plain") == 0.0


def test_code_reward_sandbox():
    good = "```python\ndef solution(a, b):\n    return a + b\n```"
    tests = [{"input": "[1, 2]", "expected_output": "3"}, {"input": "[2, 2]", "expected_output": "5"}]
    assert code_reward(good, tests) == 0.5
    evil = "```python\nimport os\ndef solution(a, b):\n    return os.getcwd()\n```"
    assert code_reward(evil, tests) == 0.0
    sneaky = "```python\ndef solution(a, b):\n    return open('/etc/passwd').read()\n```"
    assert code_reward(sneaky, tests) == 0.0
    assert code_reward("no code", tests) == 0.0


def test_length_thinking_and_combined():
    assert length_penalty("w " * 25, min_words=50) == 0.5
    assert length_penalty("w " * 512) == pytest.approx(1.0)
    assert length_penalty("w " * 5000) == 0.5
    assert thinking_quality_reward("nothing") == 0.0
    assert thinking_quality_reward("<think>" + "x" * 150 + "</think><answer>1</answer>") == pytest.approx(0.9)
    calc = RewardCalculator()
    r = calc.compute(r"<think>t</think><answer>\boxed{2}</answer>", "combined",
                     reward_weights={"math": 0.5, "format": 0.5}, math={"ground_truth": "2"})
    assert r == pytest.approx(1.0)
    with pytest.raises(ValueError):
        calc.compute("x", "nope")
    assert calc.batch(["<think>a</think><answer>b</answer>", "x"], "format") == [1.0, 0.0]


@pytest.fixture(scope="module")
def tiny():
    torch.manual_seed(0)
    cfg = MamformerConfig.from_preset("debug")
    return MamformerForCausalLM(cfg).eval(), MamformerTokenizer()


def test_reflection_module_shapes_and_loss(tiny):
    model, _ = tiny
    rm = ReflectionModule(256, 1000, embedding_weight=model.model.embed_tokens.weight)
    h = torch.randn(2, 12, 256)
    toks = torch.randint(0, 1000, (2, 5))
    out = rm(h, toks)
    assert out["refined_logits"].shape == (2, 12, 1000) and out["critique_logits"].shape == (2, 1, 1000)
    assert out["confidence"].shape == (2, 1)
    labels = torch.randint(0, 1000, (2, 12))
    loss, aux = rm.compute_reflection_loss(torch.randn(2, 12, 1000), out["refined_logits"], labels, out["confidence"])
    loss.backward()
    assert rm.refine_weight.grad is not None and 0 <= float(aux["improvement_rate"]) <= 1
    m2 = add_reflection_to_model(MamformerForCausalLM(MamformerConfig.from_preset("debug")), 1000)
    assert isinstance(m2.reflection, ReflectionModule)


def test_self_reflective_generator(tiny):
    model, tok = tiny
    rm = ReflectionModule(256, 1000)
    gen = SelfReflectiveGenerator(model, rm, tok)
    ids = torch.randint(3, 200, (1, 6))
    out, info = gen.generate_with_reflection(ids, max_new_tokens=4, reflection_threshold=0.0)
    assert info["used_reflection"] and out.shape[0] == 1 and out.shape[1] > 6


def test_chat_session_roundtrip(tiny, tmp_path):
    model, tok = tiny
    s = ChatSession(model, tok, system_prompt="Be brief.", max_context=256, template=SIMPLE_CHAT_TEMPLATE)
    s.max_new_tokens = 4
    s.add_user_message("hi")
    r = s.generate_response()
    assert isinstance(r, str) and s.get_history()[-1]["role"] == "assistant"
    s.add_user_message("x " * 300)
    s._trim_to_context()
    assert s.get_system_prompt() == "Be brief."
    p = tmp_path / "chat.json"
    s.save(str(p))
    s2 = ChatSession.load(str(p), model, tok)
    assert s2.get_history() == s.get_history() and s2.max_new_tokens == 4
    assert ChatSession._parse_thinking_response("<thinking>a</thinking>\n<answer>b") == ("a", "b")
    assert ChatSession._parse_critique_response("<draft>x</draft><final>y</final>") == "y"
    c = create_chat(model, tok, system_prompt="s")
    assert c.max_context == model.config.generation.max_context
    s.reflection_mode = "think"
    s.think_tokens = 2
    s.add_user_message("q")
    assert isinstance(s.generate_with_reflection(), str)


def test_chat_stream(tiny):
    model, tok = tiny
    s = ChatSession(model, tok, max_context=256)
    s.max_new_tokens = 3
    s.add_user_message("hello")
    chunks = list(s.generate_stream())
    assert 1 <= len(chunks) <= 3


def test_checkpoint_roundtrip_and_resume(tmp_path):
    from mamformer_b200.checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
    from mamformer_b200.engine import TrainConfig, Trainer
    cfg = MamformerConfig.from_preset("debug")
    torch.manual_seed(0)
    tr = Trainer(MamformerForCausalLM(cfg), TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=2,
                                                        compute_dtype=torch.float32))
    ids = torch.randint(0, 1000, (2, 16))
    tr.train_step(ids)
    path = save_checkpoint(str(tmp_path / "checkpoint_step_1.pt"), tr.model, tr.optimizer, tr.scheduler, step=1)
    ck = torch.load(path, weights_only=False)
    assert ck["step"] == 1 and all(v.dtype in (torch.float32, torch.int64) for v in ck["model"].values())
    masters = {}
    for _, seg in tr.optimizer.segments:
        for p, o in zip(seg.params, seg.offsets):
            masters[id(p)] = seg.master[o:o + p.numel()].view(p.shape).clone()
    ref = {n: masters[id(p)] for n, p in tr.model.named_parameters()}
    torch.manual_seed(1)
    tr2 = Trainer(MamformerForCausalLM(cfg), TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=2,
                                                         compute_dtype=torch.float32))
    step = load_checkpoint(path, tr2.model, tr2.optimizer, tr2.scheduler)
    assert step == 1 and latest_checkpoint(str(tmp_path)) == path
    got = {}
    for _, seg in tr2.optimizer.segments:
        for p, o in zip(seg.params, seg.offsets):
            got[id(p)] = seg.master[o:o + p.numel()].view(p.shape)
    for n, p in tr2.model.named_parameters():
        assert torch.equal(got[id(p)], ref[n]), n
        assert torch.equal(p.detach().float(), ref[n].to(p.dtype).float()), n
    l1 = float(tr.train_step(ids, sync_loss=True))
    l2 = float(tr2.train_step(ids, sync_loss=True))
    assert abs(l1 - l2) < 1e-6


def test_grpo_step_cpu():
    from mamformer_b200.grpo import (GRPOConfig, GRPOTrainer, PromptDataset, collate_prompts, compute_grpo_loss,
                                     group_advantages, rollout_temperatures)
    from mamformer_b200.sgrpo import StochasticGRPOConfig
    a = group_advantages(torch.tensor([[1.0, 0.0, 1.0, 0.0]]))
    assert torch.allclose(a.mean(), torch.tensor(0.0)) and a[0, 0] > 0
    assert rollout_temperatures(1.0, 3) == [0.9, 1.0, 1.1]
    loss, m = compute_grpo_loss(torch.tensor([[-1.0, -2.0]]), torch.tensor([[-1.0, -1.0]]), torch.tensor([[1.0, -1.0]]))
    assert float(loss) == pytest.approx(-0.5 + 0.04 * 0.5)
    tok = MamformerTokenizer()
    ds = PromptDataset("/nonexistent.jsonl", tok)
    batch = collate_prompts([ds[0], ds[1]])
    torch.manual_seed(0)
    policy = MamformerForCausalLM(MamformerConfig.from_preset("debug"))
    tr = GRPOTrainer(policy, tok, GRPOConfig(group_size=2, gen_max_tokens=4, learning_rate=1e-4,
                                             sgrpo=StochasticGRPOConfig(enabled=True, p=0.5, seed=0)))
    before = [p.detach().clone() for p in tr.policy.parameters()]
    m = tr.step(batch)
    assert torch.isfinite(m["loss"]) and tr.global_step == 1
    assert any(not torch.equal(b, p.detach()) for b, p in zip(before, tr.policy.parameters()))


def test_thinking_controller_phases_and_events():
    from mamformer_b200.thinking import MultiPathController, ThinkingConfig, ThinkingMode
    tc = ThinkingConfig.from_preset("FastThink", budget=3)
    assert tc.is_active and tc.effective_num_paths == 2 and tc.effective_budget == 3
    assert tc.effective_summary_budget == ThinkingMode.FastThink.default_summary_budget == 64
    assert tc.total_think_budget == 6 and "paths=2" in tc.summary()
    ctl = MultiPathController(tc)
    assert ctl.phase == "prompt" and not ctl.path_done
    ctl.start_path(0)
    assert ctl.phase == "path:0" and not ctl.path_done
    assert ctl.record_path_token(0, 11) is None
    assert ctl.record_path_token(0, tc.think_end_token_id) == "end_path"
    assert ctl.phase == "between_paths" and ctl.path_done
    ctl.start_path(1)
    assert [ctl.record_path_token(1, t) for t in (20, 21, 22)] == [None, None, "budget_exceeded"]
    assert ctl.record_path_token(1, tc.think_end_token_id) == "end_path" and ctl.phase == "paths_done"
    ctl.start_summary()
    assert not ctl.summary_done
    for i in range(63):
        assert ctl.record_summary_token(100 + i) is None
    assert ctl.record_summary_token(999) == "end_summary" and ctl.summary_done
    ctl.start_answer()
    assert ctl.record_answer_token(7) is None and not ctl.answer_done
    assert ctl.record_answer_token(2) == "end_answer" and ctl.is_done
    out = ctl.finalize()
    assert out["all_paths"] == [[11, 4], [20, 21, 22, 4]]
    assert out["path_counts"] == [1, 3] and out["path_budget_forced"] == [False, True]
    assert out["summary_count"] == 64 and out["summary_budget_forced"]
    assert out["answer_tokens"] == [7] and out["total_think_tokens"] == 4 and out["phase"] == "done"
    # an answer token before the answer phase is a caller bug
    bad = MultiPathController(tc)
    bad.start_path(0)
    with pytest.raises(RuntimeError):
        bad.record_answer_token(2)
    with pytest.raises(ValueError):
        ThinkingConfig(num_paths=-1).validate()
    with pytest.raises(ValueError):
        ThinkingMode.from_string("UltraThink")
