"""Device sampler and infer_ffi (GPU).

The sampler is held to the bit: on the same logits its id and the
probabilities it leaves in the logits row equal the Python restatement of
sampler.rs (oracle/tokenizer_ref.py), call after call (the top-p path keeps
the reference's persistent, re-sorted probability array). infer_ffi is
checked against the console's loop (main.rs:186-214) run on the host over the
device forward: the same prompt tokens, the restated sampler on the device's
logits, the pieces decoded one by one; with temperature 0 the greedy ids are
also checked against the CPU oracle's own forward."""
from __future__ import annotations

import numpy as np
import pytest

import tokenizer_files as tf
import tokenizer_ref as tr

pytestmark = pytest.mark.gpu


def _logits(rng, V, scale):
    return (rng.standard_normal(V) * scale).astype(np.float32)


@pytest.mark.parametrize("V", [1000, 128256])
@pytest.mark.parametrize("temp,top_p", [(0.0, 0.9), (0.7, 0.9), (1.0, 1.0), (0.8, 0.0), (1.3, 0.5), (0.5, 0.999)])
def test_sampler_matches_restatement(yl, torch_cuda, V, temp, top_p):
    torch = torch_cuda
    rng = np.random.default_rng(V + int(temp * 10) + int(top_p * 100))
    ours = yl.Sampler(V, temp, top_p, 42)
    ref = tr.Sampler(V, temp, top_p, 42)
    for step in range(5):
        # flat and peaked distributions, so the kept set grows and shrinks
        # (the leftovers of earlier calls take part in the next sort)
        x = _logits(rng, V, [0.5, 4.0, 1.0, 8.0, 0.1][step])
        d = torch.from_numpy(x).cuda()
        got = ours.sample(d)
        want = ref.sample(x.copy())
        assert got == want, (step, got, want)
        if temp != 0.0:  # the row now holds the probabilities, as in the reference
            e = tr.exp_f32(((x / np.float32(temp)).astype(np.float32) -
                            (x / np.float32(temp)).astype(np.float32).max()).astype(np.float32))
            p = (e / np.add.accumulate(e, dtype=np.float32)[-1]).astype(np.float32)
            assert np.array_equal(d.cpu().numpy(), p)
    ours.close()


@pytest.fixture(scope="module")
def chat_models(tmp_path_factory, yl):
    root = tmp_path_factory.mktemp("chat")
    vocab, merges = tf.learn_bpe(tf.corpus(5), 500)
    out = {}
    small_vocab = vocab + [f"<|pad_{i}|>" for i in range(1000 - len(vocab))]
    base = yl.synth_preset("tiny128", str(root / "base_small.gguf"))
    out["small"] = tf.retokenize_gguf(base, root / "small.gguf", small_vocab, merges, 1, 2, pre="gpt2")
    # the same models carrying chat templates (GGUF tokenizer.chat_template)
    tmpl_vocab = vocab + ["<|im_start|>", "<|im_end|>"] + [f"<|pad_{i}|>" for i in range(998 - len(vocab))]
    out["small_tmpl"] = tf.retokenize_gguf(base, root / "small_tmpl.gguf", tmpl_vocab, merges, 1, 2, pre="gpt2",
                                           template=BLOCKS_TEMPLATE)
    base = yl.synth_preset("tiny128", str(root / "base_big.gguf"), vocab_size=128256)
    out["llama"] = tf.retokenize_gguf(base, root / "llama.gguf", tf.llama_vocab(vocab), merges, 128000, 128009,
                                      pre="gpt2")
    out["llama_tmpl"] = tf.retokenize_gguf(base, root / "llama_tmpl.gguf", tf.llama_vocab(vocab), merges, 128000,
                                           128009, pre="gpt2", template=HEADERS_TEMPLATE)
    return out


BLOCKS_TEMPLATE = """{%- for m in messages -%}
<|im_start|>{{ m.role }}
{{ m.content }}<|im_end|>
{% endfor -%}
{%- if add_generation_prompt %}<|im_start|>assistant
{% endif %}"""

HEADERS_TEMPLATE = """{%- for m in messages %}
    {{- '<|start_header_id|>' + m['role'] + '<|end_header_id|>\n\n' + m['content'] | trim + '<|eot_id|>' }}
{%- endfor %}
{%- if add_generation_prompt %}{{ '<|start_header_id|>assistant<|end_header_id|>\n\n' }}{% endif %}"""


def host_console_loop(yl, path, prompt, temp, top_p, seed, max_tokens):
    """main.rs:186-214 on the host: device forward, restated sampler."""
    m = yl.load_transformer(path)
    tok = m.tokenizer()
    ids = tok.chat_prompt(prompt)
    assert ids == tr.Tokenizer.from_gguf(path).chat_prompt(prompt)
    s = m.create_session()
    smp = tr.Sampler(m.vocab_size(), temp, top_p, seed)
    lg, _ = m.forward_x_full(ids, 0, s)
    nxt = smp.sample(lg)
    pos, gen, reply, toks = len(ids), 0, "", []
    while nxt != m.eos_token() and pos < m.max_ctx_len() and gen < max_tokens:
        reply += tok.decode([nxt])
        toks.append(nxt)
        lg, _ = m.forward_x_full([nxt], pos, s)
        pos += 1
        gen += 1
        nxt = smp.sample(lg)
    s.close()
    m.close()
    return reply, ids, toks


@pytest.mark.parametrize("kind", ["small", "llama", "small_tmpl", "llama_tmpl"])
def test_infer_ffi_matches_console_loop(yl, torch_cuda, chat_models, kind):
    path = chat_models[kind]
    assert yl.load_transformer_ffi(path)
    for prompt, temp, top_p in [("hello world", 0.7, 0.9), ("what's 3.14?", 1.0, 1.0), ("kalo mi", 0.0, 0.9)]:
        yl.infer_config(temp, top_p, 42, 24)
        got = yl.infer_ffi(prompt)
        want, _, _ = host_console_loop(yl, path, prompt, temp, top_p, 42, 24)
        assert got == want, (kind, prompt, got, want)
    assert yl.infer_ffi("") is None  # empty prompt: NULL, no abort
    assert yl.infer_ffi(" \t\n") is None  # empty once trimmed (the console skips the line)
    yl.infer_config(0.0, 0.9, 42, 8)  # greedy: the same reply whatever the sampler's state
    assert yl.infer_ffi(" \thello world\n") == yl.infer_ffi("hello world")  # trimmed as main.rs:173


def test_infer_ffi_greedy_matches_oracle(yl, orc, torch_cuda, chat_models):
    """Temperature 0: the generated ids equal the CPU oracle's greedy ids."""
    path = chat_models["small"]
    assert yl.load_transformer_ffi(path)
    yl.infer_config(0.0, 0.9, 42, 16)
    got = yl.infer_ffi("hello world")
    _, ids, toks = host_console_loop(yl, path, "hello world", 0.0, 0.9, 42, 16)
    om = orc.Model(path, 512)
    os_ = om.create_session()
    lo = om.forward_x(ids, 0, os_)
    pos, oracle_ids = len(ids), []
    nxt = orc.argmax(lo)
    while len(oracle_ids) < 16 and nxt != 2:
        oracle_ids.append(nxt)
        lo = om.forward_x([nxt], pos, os_)
        pos += 1
        nxt = orc.argmax(lo)
    assert toks == oracle_ids
    tok = tr.Tokenizer.from_gguf(path)
    assert got == "".join(tok.decode([t]) for t in oracle_ids)
