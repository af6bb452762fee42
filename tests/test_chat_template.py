"""Chat templates (CPU): the product's C++ renderer through the C-ABI against
jinja2 set to minijinja's defaults (oracle/tokenizer_ref.py; the reference
renders with minijinja, tokenizer.rs:408-430), on templates written for these
tests in the shapes chat templates take, and the token level
(render_chat_template + encode_template_output, the console's prompt with a
template) against the restatement of tokenizer.rs:418-508."""
from __future__ import annotations

import pytest

import tokenizer_files as tf
import tokenizer_ref as tr

FORMAT, UNSUPPORTED = -3, -8

# turn markers in the ChatML style, one message per block
T_BLOCKS = """{%- for m in messages -%}
<|im_start|>{{ m.role }}
{{ m.content }}<|im_end|>
{% endfor -%}
{%- if add_generation_prompt %}<|im_start|>assistant
{% endif %}
"""

# header style: a leading system message pulled out, the rest sliced off it
T_HEADERS = """{{- bos_token }}
{%- if messages[0]['role'] == 'system' %}
    {%- set sys = messages[0]['content'] | trim %}
    {%- set rest = messages[1:] %}
{%- else %}
    {%- set sys = "" %}
    {%- set rest = messages %}
{%- endif %}
{%- if sys %}<|start_header_id|>system<|end_header_id|>

{{ sys }}<|eot_id|>{% endif %}
{%- for m in rest %}
    {{- '<|start_header_id|>' + m['role'] + '<|end_header_id|>\\n\\n' + m['content'] | trim + '<|eot_id|>' }}
{%- endfor %}
{%- if add_generation_prompt %}{{ '<|start_header_id|>assistant<|end_header_id|>\\n\\n' }}{% endif %}
"""

# the same, with nothing after the last message: the console drops its <|eot_id|>
T_HEADERS_NO_GEN = """{%- for m in messages -%}
<|start_header_id|>{{ m.role }}<|end_header_id|>

{{ m.content }}<|eot_id|>
{%- endfor %}"""

# expressions: namespaces, loop variables, filters, tests, arithmetic, slices
T_EXPR = """{%- set ns = namespace(n=0, seen=false) -%}
{%- for m in messages if m.role != 'tool' -%}
{%- set ns.n = ns.n + 1 -%}
[{{ loop.index }}/{{ loop.length }}{{ ' last' if loop.last else '' }}{{ ' first' if loop.first }}] {{ m.role | upper }}: {{ m.content | replace('a', 'A') }}
{% if 'x' in m.content %}{% set ns.seen = true %}{% endif -%}
{%- endfor -%}
count={{ ns.n }} seen={{ ns.seen }} roles={{ messages | map(attribute='role') | join(',') }}
users={{ messages | selectattr('role', 'equalto', 'user') | list | length }} others={{ messages | rejectattr('role', 'eq', 'user') | list | length }}
{{ (messages | first).role }}-{{ (messages | last).role }} {{ undefined_thing | default('dflt') }} {{ '' | default('e', true) }}
{%- for i in range(3) %} {{ i * 2 // 3 }}{{ '-' if i is odd else '+' }}{% endfor %}
{{ 'abcdef'[::-2] }} {{ 'abcdef'[1:4] }} {{ 'abcdef'[-2:] }} {{ [1, 2, 3][::-1] | join }} {{ 17 % 5 }} {{ -17 // 5 }} {{ 2 ** 5 }} {{ -(3) | abs }}
{%- if messages | length is divisibleby 2 %} even{% else %} odd{% endif %}
{%- for k, v in (messages[0] | items) %} {{ k }}={{ v | length }}{% endfor %}
{{ 'ab' ~ 3 ~ 'cd' }} {{ "x" * 3 }} {{ 'a' 'b' }} {{ "t\\tq\\u00e9\\\\" }} {{ messages[0].content[0] }} {{ 'é日本'[1] }}
{%- for c in 'hé' %}<{{ c }}>{% endfor %} {{ 'Hello World' | lower }} {{ 'hello' | capitalize }} {{ [3, 1, 2] | reverse | list | join('.') }}
{{ messages | map(attribute='role') | select('equalto', 'user') | list | length }} {{ 'b' in ['a', 'b'] }} {{ 'z' not in 'abc' }} {{ 3 > 2 and 'yes' or 'no' }}
{%- if messages[-1].role is string and messages[-1].nothing is undefined and not messages[-1].nothing is defined %} ok{% endif %}
{%- for x in [] %}never{% else %} empty-loop{% endfor %}
{%- for a in [1, 2] %}{% for b in 'xy' %} {{ loop.depth }}{{ a }}{{ b }}{{ loop.previtem | default('^') }}{{ loop.nextitem | default('$') }}{% endfor %}{% endfor %}
{{ {'k': 'v', 'j': 1}['k'] }} {{ {'k': 1} | length }} {{ (1, 2) | length }} {{ 'abc' | list | first }} {{ '  pad  ' | trim }}|{{ 'xxhixx' | trim('x') }}
"""

# whitespace control, comments, trailing newlines
T_SPACE = """  head  {#- a comment -#}  {{- ' x ' -}}  mid {# kept #} {%- if true +%}   in   {%- endif -%}   tail
{{ messages | length }}

"""

MSGS = [
    ([("user", "hi")], True),
    ([("system", "  be brief \n"), ("user", "what's 2+2? x"), ("assistant", "4"),
      ("user", "and  é日本 ")], True),
    ([("system", "  be brief \n"), ("user", "what's 2+2? x"), ("assistant", "4"),
      ("user", "and  é日本 ")], False),
    ([("user", "hello"), ("assistant", "")], True),  # the console's turn (tokenizer.rs:496-505)
    ([("tool", "a tool said x"), ("user", "ok")], False),
    ([], True),
]


def _both(yl, template, msgs, gen):
    try:
        want, werr = tr.render_chat_template_text(template, msgs, gen), None
    except Exception as e:  # noqa: BLE001 - any jinja2 error means the render fails
        want, werr = None, e
    try:
        got, gerr = yl.render_chat_template(template, msgs, gen), None
    except yl.YlError as e:
        got, gerr = None, e
    if werr is not None:
        assert gerr is not None and gerr.code == FORMAT, (template, msgs, werr, got)
    else:
        assert gerr is None, (gerr, want)
        assert got == want, (msgs, got, want)
    return got


@pytest.mark.parametrize("name", ["blocks", "headers", "headers_no_gen", "expr", "space"])
def test_render_matches_jinja(yl, name):
    template = {"blocks": T_BLOCKS, "headers": T_HEADERS, "headers_no_gen": T_HEADERS_NO_GEN, "expr": T_EXPR,
                "space": T_SPACE}[name]
    rendered = [_both(yl, template, msgs, gen) for msgs, gen in MSGS]
    assert sum(r is not None and r != "" for r in rendered) >= 4  # most cases render something


@pytest.mark.parametrize("template", [
    "{% for m in messages %}{{ loop.cycle('odd', 'even') }}-{{ loop.cycle(1, 2, 3) }} {% endfor %}",
    "a {% raw %}{{ x }} {% if %}{# c #}{% endraw %} b",
    "a {%- raw -%}  {{ y }}  {%- endraw -%}  b",
    "{% raw %}{% endraw %}|{% raw %} {% endraw %}|",
    "{% for m in messages %}{% raw %}<{{ m }}>{% endraw %}{{ m.role }}{% endfor %}",
    "x {% raw %}  {%- if -%}  {% endraw -%}   y",  # markers inside the raw text are text
])
def test_raw_blocks_match_jinja(yl, template):
    _both(yl, template, [("user", "hi"), ("assistant", "ok"), ("user", "again")], True)


def test_render_known_values(yl):
    r = yl.render_chat_template(T_BLOCKS, [("user", "hi")], True)
    assert r == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    assert yl.render_chat_template("abc\n", [], False) == "abc"  # one trailing newline dropped
    assert yl.render_chat_template("abc\n\n", [], False) == "abc\n"
    assert yl.render_chat_template("{{ x }}|{{ true }}|{{ none }}|{{ 3 }}", [], False) == "|true|none|3"
    assert yl.render_chat_template("{{ '}}' }}{{ \"%}\" }}", [], False) == "}}%}"
    # a set inside a loop lasts for the loop (minijinja's one loop frame), not after it
    t = "{% for i in [1, 2] %}{% if i == 2 %}{{ x }}{% endif %}{% set x = i %}{% endfor %}[{{ x }}]"
    assert yl.render_chat_template(t, [], False) == "1[]"


@pytest.mark.parametrize("template,code", [
    ("{{ bos_token + 'x' }}", FORMAT),               # arithmetic on an undefined value
    ("{{ messages[0].content.strip() }}", FORMAT),   # no Python string methods in minijinja
    ("{{ raise_exception('no') }}", FORMAT),         # an undefined function
    ("{{ nothing.attr }}", FORMAT),                  # attribute of an undefined value
    ("{{ messages | nonexistent }}", FORMAT),        # unknown filter
    ("{% if true %}open", FORMAT),                   # missing endif
    ("{% endfor %}", FORMAT),
    ("{{ 1 + }}", FORMAT),
    ("{{ 'unterminated }}", FORMAT),
    ("{% frobnicate %}", FORMAT),
    ("{{ 1.5 }}", UNSUPPORTED),
    ("{{ 7 / 2 }}", UNSUPPORTED),
    ("{% macro f() %}x{% endmacro %}{{ f() }}", UNSUPPORTED),
    ("{{ messages | tojson }}", UNSUPPORTED),
    ("{% raw %}never closed", FORMAT),
    ("{% endraw %}", FORMAT),
    ("{{ 'É' | lower }}", UNSUPPORTED),
])
def test_render_errors(yl, template, code):
    msgs = [("user", "hi")]
    with pytest.raises(yl.YlError) as ei:
        yl.render_chat_template(template, msgs, True)
    assert ei.value.code == code, ei.value
    if code == FORMAT:  # jinja2 (set to minijinja's defaults) fails these too
        with pytest.raises(Exception):
            tr.render_chat_template_text(template, msgs, True)


def test_render_bounds_nesting(yl):
    """Template text comes from model files: nesting that would exhaust a thread's stack fails cleanly."""
    msgs = [("user", "hi")]
    deep = [
        "{{ " + "(" * 5000 + "1" + ")" * 5000 + " }}",
        "{{ " + "-" * 5000 + "1 }}",
        "{{ " + "not " * 5000 + "true }}",
        "{{ " + " ~ ".join(["'a'"] * 3000) + " }}",
        "{{ 'a'" + " | trim" * 3000 + " }}",
        "{% if true %}" * 300 + "x" + "{% endif %}" * 300,
    ]
    for t in deep:
        with pytest.raises(yl.YlError) as ei:
            yl.render_chat_template(t, msgs, True)
        assert ei.value.code == FORMAT
        assert "too deep" in str(ei.value)  # the message reaches the calling thread
    # well inside the limits
    assert yl.render_chat_template("{{ " + "(" * 150 + "1" + ")" * 150 + " }}", msgs, True) == "1"
    assert yl.render_chat_template("{% if true %}" * 150 + "x" + "{% endif %}" * 150, msgs, True) == "x"
    assert yl.render_chat_template("{{ " + " ~ ".join(["'a'"] * 900) + " }}", msgs, True) == "a" * 900


def test_render_on_a_small_thread_stack(tmp_path):
    """Parsing and rendering run on a thread of their own: templates at the
    nesting limits render from a caller thread with a 128 KiB stack."""
    import subprocess
    import sys
    from pathlib import Path
    script = tmp_path / "small_stack.py"
    script.write_text(f"""
import sys, threading
sys.path.insert(0, {str(Path(__file__).parent)!r})
from conftest import load_package
yl = load_package()
threading.stack_size(128 * 1024)
m = [("user", "hi")]
T = ["{{{{ " + "(" * 249 + "1" + ")" * 249 + " }}}}",
     "{{{{ " + " ~ ".join(["'a'"] * 999) + " }}}}",
     "{{% if true %}}" * 200 + "x" + "{{% endif %}}" * 200,
     "{{{{ 'a'" + " | trim" * 999 + " }}}}"]
out = []
t = threading.Thread(target=lambda: out.extend(len(yl.render_chat_template(x, m, True)) for x in T))
t.start()
t.join()
print(out)
""")
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == "[1, 999, 1, 1]"


def test_render_rejects_non_utf8_message(yl):
    import ctypes as C
    lib = yl.raw_lib()
    roles = (C.c_char_p * 1)(b"user")
    contents = (C.c_char_p * 1)(b"\xff\xfe")
    n = C.c_uint64()
    buf = C.create_string_buffer(64)
    rc = lib.yl_chat_template_render(b"{{ messages[0].content }}", C.cast(roles, C.c_void_p),
                                     C.cast(contents, C.c_void_p), 1, 1, buf, 64, C.byref(n))
    assert rc == -1  # YL_ERR_ARG


@pytest.fixture(scope="module")
def bpe():
    return tf.learn_bpe(tf.corpus(7), 400)


def test_template_prompt_small_vocab(yl, tmp_path, bpe):
    vocab, merges = bpe
    specials = ["<|im_start|>", "<|im_end|>"]
    path = tf.write_gguf_tokenizer(tmp_path / "s.gguf", vocab + specials, merges, 1, 2, add_bos=True,
                                   template=T_BLOCKS)
    ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)
    assert ours.info()["has_template"]
    start = len(vocab)
    for user in ["hello world", "what's <b>bold</b> 3.14?", "日本 <|im_end|> inside"]:
        p = ours.chat_prompt(user)
        assert p == ref.chat_prompt(user), user
        assert p[0] == 1 and p[1] == start  # BOS, then <|im_start|> as one id
        assert ours.chat_prompt(user, system="be brief") == ref.chat_prompt(user, system="be brief")
    for msgs, gen in MSGS:
        assert ours.render_chat(msgs, gen) == ref.render_chat(msgs, gen), msgs


def test_template_prompt_llama_vocab(yl, tmp_path, bpe):
    vocab, merges = bpe
    big = tf.llama_vocab(vocab)
    for name, template in (("h", T_HEADERS), ("n", T_HEADERS_NO_GEN)):
        path = tf.write_gguf_tokenizer(tmp_path / f"{name}.gguf", big, merges, 128000, 128009, template=template)
        ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)
        for user in ["hi", "what's <|eot_id|> 2+2?"]:
            p = ours.chat_prompt(user)
            assert p == ref.chat_prompt(user)
            assert p[0] == 128000 and p.count(128006) >= 1
            if template is T_HEADERS_NO_GEN:  # the empty assistant turn's <|eot_id|> is dropped
                assert p[-1] != 128009
                assert p.count(128009) == 1 + user.count("<|eot_id|>")  # the user turn's own one stays
            else:  # ends on the generation prompt's header
                tail = [128006] + ref.encode("assistant") + [128007] + ref.encode("\n\n")
                assert p[-len(tail):] == tail


def test_encode_template_output_longest_match(yl, tmp_path, bpe):
    vocab, merges = bpe
    # duplicate texts (the later id wins), nested prefixes, a '<' entry that is not a prefix anywhere
    extra = ["<|a|>", "<|a|>b", "<|a|>", "<|", "x<y"]
    path = tf.write_gguf_tokenizer(tmp_path / "e.gguf", vocab + extra, merges, 1, 2,
                                   template="{% for m in messages %}{{ m.content }}{% endfor %}")
    ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)
    base = len(vocab)
    for text in ["x<|a|>b<|a|>c<y<|", "<|a|><|a|>bb", "plain text", "<", "<<|", "a<b <c", "<|a"]:
        got = ours.render_chat([("user", text)], False)
        assert got == ref.render_chat([("user", text)], False), text
    got = ours.render_chat([("user", "<|a|>b<|a|>")], False)
    assert got == [base + 1, base + 2]
    assert ours.render_chat([], False) == []  # empty render: no ids


def test_encode_template_output_fuzz(yl, tmp_path, bpe):
    """Random texts dense in '<', special-token fragments and near misses:
    the indexed longest match equals the literal scan of every entry."""
    import random
    vocab, merges = bpe
    extra = ["<|im_start|>", "<|im_end|>", "<|im", "<|", "<s>", "</s>", "<s", "<|im_start|>x", "<|im_end|>"]
    path = tf.write_gguf_tokenizer(tmp_path / "f.gguf", vocab + extra, merges, 1, 2,
                                   template="{% for m in messages %}{{ m.content }}{% endfor %}")
    ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)
    r = random.Random(11)
    pieces = extra + ["<", "<<", "|", ">", "im", " ", "\n", "hello", "é", "日本", "x", "/s", "s>", "<|im_st"]
    for _ in range(150):
        text = "".join(r.choice(pieces) for _ in range(r.randint(1, 14)))
        assert ours.render_chat([("user", text)], False) == ref.render_chat([("user", text)], False), text


def test_template_that_does_not_parse(yl, tmp_path, bpe):
    vocab, merges = bpe
    path = tf.write_gguf_tokenizer(tmp_path / "b.gguf", vocab, merges, 1, 2, template="{% if %}")
    t = yl.Tokenizer.load(path)  # loads; encode and decode still work
    assert t.decode(t.encode("hello")) == "hello"
    with pytest.raises(yl.YlError) as ei:
        t.chat_prompt("hi")
    assert ei.value.code == FORMAT
    path = tf.write_gguf_tokenizer(tmp_path / "u.gguf", vocab, merges, 1, 2, template="{% macro m() %}{% endmacro %}")
    with pytest.raises(yl.YlError) as ei:
        yl.Tokenizer.load(path).chat_prompt("hi")
    assert ei.value.code == UNSUPPORTED


def test_no_template_unchanged(yl, tmp_path, bpe):
    vocab, merges = bpe
    path = tf.write_gguf_tokenizer(tmp_path / "n.gguf", vocab, merges, 1, 2)
    t = yl.Tokenizer.load(path)
    assert not t.info()["has_template"]
    assert t.render_chat([("user", "hi")], True) == []  # render_chat_template without a template


# ------------------------------------------------------- random expressions --
# Typed random expressions (ints, ASCII strings, booleans, lists of ints) in
# the operators, filters and tests above, rendered by both engines; values
# stay small, so arithmetic never overflows, and no case relies on the few
# places where jinja2 and minijinja differ (bool arithmetic, float division,
# printing lists).

class _Gen:
    WORDS = ["", "a", "ab", "Abc", " pad ", "x y", "hello", "AaA", "z"]

    def __init__(self, seed):
        import random
        self.r = random.Random(seed)

    def pick(self, *fs):
        return self.r.choice(fs)()

    def int_(self, d=0):
        r = self.r
        if d > 2:
            return str(r.randint(0, 20))
        return self.pick(
            lambda: str(r.randint(0, 20)),
            lambda: f"({self.int_(d + 1)} + {self.int_(d + 1)})",
            lambda: f"({self.int_(d + 1)} - {self.int_(d + 1)})",
            lambda: f"({self.int_(d + 1)} * {self.int_(d + 1)})",
            lambda: f"({self.int_(d + 1)} // {r.choice([1, 2, 3, -4, 7])})",
            lambda: f"({self.int_(d + 1)} % {r.choice([2, 3, 5, -3])})",
            lambda: f"-{r.randint(0, 9)}",
            lambda: f"({self.str_(d + 1)} | length)",
            lambda: f"({self.list_(d + 1)} | length)",
            lambda: f"({self.int_(d + 1)} if {self.bool_(d + 1)} else {self.int_(d + 1)})",
            lambda: "ns.n",
            lambda: f"messages | length",
            lambda: f"({self.int_(d + 1)} | abs)",
            lambda: f"([{self.int_(d + 1)}, 5] | first)",
            lambda: f"([4, {self.int_(d + 1)}] | last)",
        )

    def str_(self, d=0):
        r = self.r
        lit = lambda: repr(r.choice(self.WORDS))  # noqa: E731
        if d > 2:
            return lit()
        return self.pick(
            lit,
            lambda: f"({self.str_(d + 1)} ~ {self.str_(d + 1)})",
            lambda: f"({self.str_(d + 1)} + {self.str_(d + 1)})",
            lambda: f"({self.str_(d + 1)} ~ {self.int_(d + 1)})",
            lambda: f"({self.str_(d + 1)} | upper)",
            lambda: f"({self.str_(d + 1)} | lower)",
            lambda: f"({self.str_(d + 1)} | trim)",
            lambda: f"({self.str_(d + 1)} | capitalize)",
            lambda: f"({self.str_(d + 1)} | replace('a', 'q'))",
            lambda: f"{self.str_(d + 1)}[{r.randint(-3, 3)}:{r.choice(['', str(r.randint(-3, 5))])}]",
            lambda: f"({self.str_(d + 1)} * {r.randint(0, 3)})",
            lambda: f"({self.list_(d + 1)} | join({lit()}))",
            lambda: f"({self.str_(d + 1)} if {self.bool_(d + 1)} else {self.str_(d + 1)})",
            lambda: f"messages[{r.randint(-2, 1)}].role",
            lambda: f"messages[0]['content']",
            lambda: f"(nothing | default({lit()}))",
            lambda: f"({self.str_(d + 1)} | reverse)",
        )

    def bool_(self, d=0):
        r = self.r
        if d > 2:
            return r.choice(["true", "false"])
        cmp = lambda: r.choice(["==", "!=", "<", ">", "<=", ">="])  # noqa: E731
        return self.pick(
            lambda: r.choice(["true", "false"]),
            lambda: f"({self.int_(d + 1)} {cmp()} {self.int_(d + 1)})",
            lambda: f"({self.str_(d + 1)} {cmp()} {self.str_(d + 1)})",
            lambda: f"({self.str_(d + 1)} in {self.str_(d + 1)})",
            lambda: f"({self.int_(d + 1)} not in {self.list_(d + 1)})",
            lambda: f"(not {self.bool_(d + 1)})",
            lambda: f"({self.bool_(d + 1)} and {self.bool_(d + 1)})",
            lambda: f"({self.bool_(d + 1)} or {self.bool_(d + 1)})",
            lambda: f"({self.int_(d + 1)} is {r.choice(['odd', 'even'])})",
            lambda: f"({self.int_(d + 1)} is divisibleby {r.choice([1, 2, 3])})",
            lambda: f"(nothing is {r.choice(['defined', 'undefined'])})",
            lambda: f"({self.str_(d + 1)} is string)",
            lambda: f"(messages[0] is mapping)",
        )

    def list_(self, d=0):
        r = self.r
        if d > 2:
            return "[1, 2, 3]"
        return self.pick(
            lambda: "[" + ", ".join(self.int_(d + 1) for _ in range(r.randint(0, 3))) + "]",
            lambda: f"({self.list_(d + 1)} | reverse | list)",
            lambda: f"{self.list_(d + 1)}[{r.choice(['1:', '::-1', ':2', '-2:'])}]",
            lambda: f"({self.list_(d + 1)} + {self.list_(d + 1)})",
            lambda: f"(range({r.randint(0, 4)}) | list)",  # a Python range in jinja2, a sequence in minijinja
            lambda: f"({self.list_(d + 1)} | select('odd') | list)",
        )

    def template(self):
        r = self.r
        parts = ["{%- set ns = namespace(n=3) -%}"]
        for _ in range(r.randint(2, 5)):
            kind = r.randint(0, 5)
            if kind == 0:
                parts.append("{{ " + self.int_() + " }}|")
            elif kind == 1:
                parts.append("{{ " + self.str_() + " }}|")
            elif kind == 2:
                parts.append("{{ " + self.bool_() + " }}|")
            elif kind == 3:
                parts.append("{% if " + self.bool_() + " %}T{% elif " + self.bool_() + " %}E{% else %}F{% endif %}|")
            elif kind == 4:
                parts.append("{% for v in " + self.list_() + " %}{{ v }}{{ ',' if not loop.last }}"
                             "{% set ns.n = ns.n + v %}{% else %}none{% endfor %}|")
            else:
                parts.append("{%- set t = " + self.str_() + " -%}{{ t | length }}:{{ t }}|")
        return "".join(parts)


def test_random_expressions_match_jinja(yl):
    msgs = [("system", "sys a"), ("user", "Hi there"), ("assistant", "ok")]
    agreed = errors = 0
    for seed in range(400):
        t = _Gen(seed).template()
        try:
            want, werr = tr.render_chat_template_text(t, msgs, True), None
        except Exception as e:  # noqa: BLE001
            want, werr = None, e
        try:
            got, gerr = yl.render_chat_template(t, msgs, True), None
        except yl.YlError as e:
            got, gerr = None, e
        if werr is not None:
            assert gerr is not None and gerr.code == FORMAT, (seed, t, werr, got)
            errors += 1
        else:
            assert gerr is None and got == want, (seed, t, want, got, gerr)
            agreed += 1
    assert agreed > 300, (agreed, errors)


@pytest.mark.parametrize("big", [False, True])
def test_tokenizer_template_pieces_match_restatement(yl, tmp_path, bpe, big):
    """encode_wrap_n_header, apply_system_template, apply_turn_template (with
    and without the empty assistant turn) and set_chat_template, each against
    the restatement of tokenizer.rs:277-539, on a tokenizer without and then
    with a template."""
    vocab, merges = bpe
    if big:
        path = tf.write_gguf_tokenizer(tmp_path / "b.gguf", tf.llama_vocab(vocab), merges, 128000, 128009)
        template = T_HEADERS_NO_GEN
    else:
        path = tf.write_gguf_tokenizer(tmp_path / "s.gguf", vocab + ["<|im_start|>", "<|im_end|>"], merges, 1, 2,
                                       add_bos=True)
        template = T_BLOCKS
    ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)

    def compare():
        for text in ["hello world", "what's 3.14?", "日本 <b>"]:
            for header in ["", "system", "user"]:
                for wrap in (False, True):
                    assert ours.encode_wrap_n_header(text, header, wrap) == ref.encode_wrap_n_header(text, header, wrap)
            assert ours.apply_system_template(text) == ref.apply_system_template(text)
            for add in (False, True):
                assert ours.apply_turn_template(text, add) == ref.apply_turn_template(text, add), (text, add)
            assert ours.chat_prompt(text, system="sys") == ref.chat_prompt(text, system="sys")
        assert ours.apply_system_template("") == ref.apply_system_template("")

    compare()
    assert not ours.info()["has_template"]
    with pytest.raises(yl.YlError) as e:
        ours.set_chat_template("{% if %}")  # does not parse: the tokenizer stays as it was
    assert e.value.code == FORMAT and not ours.info()["has_template"]
    ours.set_chat_template(template)
    ref.set_chat_template(template)
    assert ours.info()["has_template"]
    compare()
