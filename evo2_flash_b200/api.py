"""The evo2_flash user surface over the B200 mixers, without an engine.

evo2_flash's `Evo2` (evo2_flash/api.py:485-982) drives a vLLM engine whose
model holds the Hyena mixers.  This module offers the same calls --
`score_sequences`, `forward` / `__call__`, `generate`, with the byte tokenizer,
`reverse_complement` and `GenerationOutput` -- on the engine-free
`StripedHyena2` harness (evo2_flash_b200.model), whose Hyena layers are this
package's mixer modules: scoring and `forward` are packed teacher-forced
prefill steps, `generate` is one prefill of the prompts followed by one-token
decode steps on the paged mixer state (the decode kernels) and the attention
key/value cache.

Kept from the reference: argument names and meanings, the scoring positions
(t >= 1, or every token after a prepended EOD), mean / sum reduction and the
reverse-complement average, vortex sampling semantics (top_k == 1 or
temperature == 0 is argmax; else temperature, top-k, then top-p over the
renormalised top-k distribution), exactly `n_tokens` generated per prompt with
EOD not stopping generation, `logprobs_mean` under the raw distribution, seed
+ i per prompt, the error messages for invalid arguments.  Not provided: the
engine arguments, checkpoint resolution and conversion, speculative decoding,
classifier-free guidance and the prefix cache, which belong to the engine.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable

import torch
import torch.nn.functional as F


class CharLevelTokenizer:
    """Byte-level tokenizer (vortex `CharLevelTokenizer(512)` semantics,
    evo2_flash/api.py:63-111): text -> its UTF-8 bytes as ids; EOD / EOS = 0,
    PAD = 1; an id decodes to chr(id) after clamping into [32, vocab_size], so
    control ids print as spaces."""

    def __init__(self, vocab_size: int = 512):
        self.name = "CharLevelTokenizer"
        self._vocab_size = int(vocab_size)
        self.eod_id = 0
        self.eos_id = 0
        self.pad_id = 1

    @property
    def vocab_size(self) -> int:
        return self._vocab_size

    @property
    def eod(self) -> int:
        return self.eod_id

    @property
    def eos(self) -> int:
        return self.eod_id

    def clamp(self, n: int) -> int:
        return min(max(int(n), 32), self._vocab_size)

    def decode_token(self, token) -> str:
        return chr(self.clamp(token))

    def tokenize(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def tokenize_batch(self, text_batch):
        if isinstance(text_batch, list):
            return [self.tokenize(t) for t in text_batch]
        return self.tokenize(text_batch)

    def detokenize(self, token_ids) -> str:
        if isinstance(token_ids, torch.Tensor):
            token_ids = token_ids.tolist()
        return "".join(self.decode_token(t) for t in token_ids)

    def detokenize_batch(self, token_ids):
        if isinstance(token_ids, torch.Tensor):
            token_ids = token_ids.tolist()
        if isinstance(token_ids, list) and token_ids and isinstance(token_ids[0], (list, tuple)):
            return [self.detokenize(t) for t in token_ids]
        return self.detokenize(token_ids)


# IUPAC nucleotide complements (Biopython's DNA table: ambiguity codes, U read as
# T); lower case maps to lower case, anything else is left as it is.
_COMPLEMENT = {"A": "T", "C": "G", "G": "C", "T": "A", "U": "A", "M": "K", "K": "M",
               "R": "Y", "Y": "R", "W": "W", "S": "S", "V": "B", "B": "V", "H": "D",
               "D": "H", "N": "N", "X": "X"}
_COMPLEMENT_TABLE = str.maketrans({**_COMPLEMENT,
                                   **{k.lower(): v.lower() for k, v in _COMPLEMENT.items()}})


def reverse_complement(seq: str) -> str:
    """The reverse complement of a DNA string (evo2_flash/api.py:118-130)."""
    return seq.translate(_COMPLEMENT_TABLE)[::-1]


@dataclass(kw_only=True)
class GenerationOutput:
    """`generate`'s result, with vortex's fields (evo2_flash/api.py:137-170).

    `logits` is computed on first access by one teacher-forced forward over
    prompt + completion: the raw logits that predicted each generated token,
    one float32 (N, n_tokens, vocab) tensor when every prompt has the same
    length and `batched`, otherwise one (1, n_tokens, vocab) tensor per prompt."""

    sequences: list[str]
    logprobs_mean: list[float]
    token_ids: list[list[int]] = field(default_factory=list, repr=False)
    _logits_fn: Callable[[], list] | None = field(default=None, repr=False)
    _logits: list | None = field(default=None, repr=False)

    @property
    def logits(self):
        if self._logits is None and self._logits_fn is not None:
            self._logits = self._logits_fn()
        return self._logits


def _sampling_args(temperature: float, top_k: int, top_p: float):
    """Validated (greedy, temperature, top_k, top_p) with vortex's meaning:
    top_k <= 0 keeps the whole vocabulary, top_p outside (0, 1) applies no
    nucleus filter, top_k == 1 or temperature == 0 is argmax."""
    if temperature < 0:
        raise ValueError(f"temperature must be >= 0, got {temperature}")
    if top_p > 1.0:
        raise ValueError("top-p should be in (0, 1].")
    greedy = top_k == 1 or temperature == 0
    return greedy, float(temperature), int(top_k), float(top_p)


def sample_token(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                 generator: torch.Generator | None = None) -> int:
    """One token from a (vocab,) logits row: argmax when top_k == 1 or
    temperature == 0; otherwise logits / temperature restricted to the top_k
    largest (top_k > 0), then to the shortest prefix of those, by decreasing
    probability, whose renormalised mass reaches top_p (0 < top_p < 1), and
    sampled from the renormalised remainder."""
    greedy, t, k, p = _sampling_args(temperature, top_k, top_p)
    x = logits.detach().float().cpu()
    if greedy:
        return int(torch.argmax(x))
    x = x / t
    order = torch.argsort(x, descending=True)
    vals = x[order]
    keep = vals.numel() if k <= 0 else min(k, vals.numel())
    vals = vals[:keep]
    probs = torch.softmax(vals, 0)
    if 0.0 < p < 1.0:
        before = torch.cumsum(probs, 0) - probs  # mass of the tokens ranked above
        probs = torch.where(before < p, probs, torch.zeros_like(probs))
        probs = probs / probs.sum()
    pick = torch.multinomial(probs, 1, generator=generator)
    return int(order[pick])


class Evo2:
    """`evo2_flash.Evo2`'s scoring, embedding and generation calls on the
    engine-free harness.

    model: a `StripedHyena2` with its weights loaded; None builds a random-init
    model of `config` (default: the 7B shape) on `device` from `seed`.
    max_tokens_per_step: the packed-step token budget (None: every prompt of a
    call in one step); longer inputs continue from the paged state.
    max_model_len: optional context limit checked like the reference's."""

    def __init__(self, model=None, *, config=None, device="cuda", seed: int = 0,
                 max_tokens_per_step: int | None = None, max_model_len: int | None = None):
        if model is None:
            from .model import StripedHyena2, StripedHyena2Config

            model = StripedHyena2(config or StripedHyena2Config.evo2_7b(), device=device)
            model.load_tensors(model.random_tensors(seed))
        self.model = model
        self.tokenizer = CharLevelTokenizer(model.cfg.vocab_size)
        self.max_tokens_per_step = max_tokens_per_step
        self.max_model_len = max_model_len

    def _check_len(self, n_tokens: int, what: str):
        if self.max_model_len is not None and n_tokens > self.max_model_len:
            raise ValueError(f"{what} needs {n_tokens} positions but "
                             f"max_model_len={self.max_model_len}")

    # ---- scoring -------------------------------------------------------------
    def score_sequences(self, seqs, batch_size: int = 1, prepend_bos: bool = False,
                        reduce_method: str = "mean",
                        average_reverse_complement: bool = False) -> list[float]:
        """Reduced log-likelihood of each sequence (evo2_flash/api.py:605-639):
        position t contributes log p(x_t | x_<t) for t >= 1, or every token
        after an EOD when `prepend_bos`; 'mean' or 'sum'; with
        `average_reverse_complement` the mean of the sequence's score and its
        reverse complement's.  `batch_size` is accepted and does not change the
        result: the sequences are packed into steps by `max_tokens_per_step`."""
        if reduce_method not in ("mean", "sum"):
            raise ValueError(f"Invalid reduce_method {reduce_method}")
        if isinstance(seqs, str):
            seqs = [seqs]
        seqs = list(seqs)
        if not seqs:
            return []
        variants = seqs + ([reverse_complement(s) for s in seqs]
                           if average_reverse_complement else [])
        bos = [self.tokenizer.eod_id] if prepend_bos else []
        ids = [bos + self.tokenizer.tokenize(s) for s in variants]
        for x in ids:
            if not x:
                raise ValueError("cannot score an empty sequence")
            self._check_len(len(x) + 1, "scoring a sequence")
        lps = self.model.token_logprobs([torch.tensor(x, dtype=torch.long) for x in ids],
                                        self.max_tokens_per_step)
        if reduce_method == "mean":  # a one-token sequence has nothing to score: NaN
            scores = [float(lp.mean()) if lp.numel() else math.nan for lp in lps]
        else:
            scores = [float(lp.sum()) for lp in lps]
        if average_reverse_complement:
            n = len(seqs)
            scores = [0.5 * (a + b) for a, b in zip(scores[:n], scores[n:])]
        return scores

    # ---- forward / embeddings -----------------------------------------------
    # vortex layer names (evo2_flash/api.py:176-192) -> what the harness captures:
    # ("embed" | "norm" | "unembed" | "block", block index) or ("module", path,
    # "out" | "in", kind restriction).  Modules are captured by forward hooks.
    _NAMES = [
        (r"embedding_layer", "embed", None, None, None),
        (r"norm", "norm", None, None, None),
        (r"unembed", "unembed", None, None, None),
        (r"blocks\.(\d+)", "block", None, None, None),
        (r"blocks\.(\d+)\.mlp", "module", "layers.{i}.mlp", "out", None),
        (r"blocks\.(\d+)\.mlp\.(l1|l2|l3)", "module", "layers.{i}.mlp.{sub}", "out", None),
        (r"blocks\.(\d+)\.projections", "module", "layers.{i}.mixer.in_proj", "out", "hyena"),
        (r"blocks\.(\d+)\.filter", "module", "layers.{i}.mixer.out_proj", "in", "hyena"),
        (r"blocks\.(\d+)\.out_filter_dense", "module", "layers.{i}.mixer.out_proj", "out",
         "hyena"),
        (r"blocks\.(\d+)\.inner_mha_cls", "module", "layers.{i}.mixer", "out", "attn"),
        (r"blocks\.(\d+)\.inner_mha_cls\.out_proj", "module", "layers.{i}.mixer.o_proj", "out",
         "attn"),
    ]

    def _resolve(self, name: str):
        """A vortex layer name -> (what, block index or None, module, "out"/"in")."""
        import re

        if re.fullmatch(r"blocks\.\d+\.(pre_norm|post_norm)", name):
            raise ValueError(f"layer name {name!r} is not supported here: this harness "
                             "applies the block norms inside the residual add (and, for "
                             "fp8 Hyena layers, inside the in_proj quantisation)")
        n_blocks = len(self.model.layers)
        for pat, what, path, io, kind in self._NAMES:
            m = re.fullmatch(pat, name)
            if not m:
                continue
            i = int(m.group(1)) if m.groups() else None
            if i is not None:
                if not 0 <= i < n_blocks:
                    raise ValueError(f"{name!r}: layer {i} out of range (model has "
                                     f"{n_blocks} blocks)")
                is_attn = self.model.layers[i].kind == "attn"
                if kind == "hyena" and is_attn:
                    raise ValueError(f"{name!r}: block {i} is an attention block; use "
                                     f"blocks.{i}.inner_mha_cls instead")
                if kind == "attn" and not is_attn:
                    raise ValueError(f"{name!r}: block {i} is a Hyena block; use "
                                     f"blocks.{i}.filter / blocks.{i}.out_filter_dense instead")
            if what != "module":
                return what, i, None, None
            target = path.format(i=i, sub=m.group(2) if len(m.groups()) > 1 else None)
            try:
                mod = self.model.get_submodule(target)
            except AttributeError:
                raise ValueError(f"layer name {name!r}: no module {target!r} in this "
                                 "model") from None
            return what, i, mod, io
        raise ValueError(f"unsupported layer name {name!r}; supported: embedding_layer, norm, "
                         "unembed, blocks.N, blocks.N.mlp[.l1|.l2|.l3], blocks.N.projections, "
                         "blocks.N.filter, blocks.N.out_filter_dense, blocks.N.inner_mha_cls"
                         "[.out_proj]")

    def forward(self, input_ids, return_embeddings: bool = False, layer_names=None):
        """(logits (B, L, vocab) bf16, embeddings dict or None), each row of
        `input_ids` an independent causal sequence (evo2_flash/api.py:764-808).
        `layer_names` are vortex names (`blocks.28.mlp.l3`, `blocks.N`, `norm`,
        ...); each embedding has shape (B, L, D) and the captured tensor's dtype,
        and 'unembed' is the logits tensor itself."""
        if return_embeddings and layer_names is None:
            raise ValueError("layer_names must be specified when return_embeddings=True")
        if isinstance(input_ids, torch.Tensor):
            rows = input_ids.detach().long().cpu()
            if rows.dim() == 1:
                rows = rows[None]
            if rows.dim() != 2:
                raise ValueError(f"input_ids must be (B, L), got shape {tuple(input_ids.shape)}")
            id_lists = rows.tolist()
        else:
            id_lists = [list(map(int, r)) for r in input_ids]
            if id_lists and not isinstance(input_ids[0], (list, tuple, torch.Tensor)):
                id_lists = [list(map(int, input_ids))]
        V = self.tokenizer.vocab_size
        for ids in id_lists:
            if len(ids) == 0:
                raise ValueError("cannot run forward on an empty sequence")
            if min(ids) < 0 or max(ids) >= V:
                raise ValueError(f"token ids must be in [0, {V})")
            self._check_len(len(ids) + 1, "forward over a sequence")
        if len({len(ids) for ids in id_lists}) > 1:
            raise ValueError("every row of input_ids must have the same length")
        names = list(layer_names or []) if return_embeddings else []
        if len(set(names)) != len(names):
            raise ValueError(f"duplicate layer names in {names}")
        specs = {n: self._resolve(n) for n in names}
        blocks = {i for what, i, _, _ in specs.values() if what == "block"}
        B, L = len(id_lists), len(id_lists[0])
        m = self.model
        logits = torch.empty(B, L, V, dtype=torch.bfloat16, device=m.device)
        emb: dict = {}
        step_caps: dict = {}

        def hook_for(name, io):
            def hook(module, args, output):
                x = args[0] if io == "in" else output
                if isinstance(x, tuple):
                    x = x[0]
                step_caps[name] = x.detach()
            return hook

        handles = [mod.register_forward_hook(hook_for(n, io))
                   for n, (what, _, mod, io) in specs.items() if what == "module"]
        seqs = [torch.tensor(x, dtype=torch.long) for x in id_lists]
        try:
            with torch.no_grad():
                for item in m.prefill_steps(seqs, self.max_tokens_per_step, blocks or None):
                    h, segs = item[0], item[1]
                    taps = item[2] if len(item) > 2 else {}
                    lg = F.linear(h, m.embed)
                    for n, (what, i, _, _) in specs.items():
                        if what == "module" and n not in step_caps:
                            raise RuntimeError(f"layer {n!r} was not captured: its module did "
                                               "not run in this step")
                        src = {"norm": h, "block": taps.get(i), "module": step_caps.get(n)}.get(what)
                        if src is None:
                            continue
                        if n not in emb:
                            emb[n] = torch.empty(B, L, *src.shape[1:], dtype=src.dtype,
                                                 device=src.device)
                    for a, b, sid, p0 in segs:
                        rows = slice(p0, p0 + (b - a))
                        logits[sid, rows] = lg[a:b]
                        for n, (what, i, _, _) in specs.items():
                            if what == "norm":
                                emb[n][sid, rows] = h[a:b]
                            elif what == "block":
                                emb[n][sid, rows] = taps[i][a:b]
                            elif what == "module":
                                emb[n][sid, rows] = step_caps[n][a:b]
                    step_caps.clear()
        finally:
            for hd in handles:
                hd.remove()
        if not return_embeddings:
            return logits, None
        for n, (what, _, _, _) in specs.items():
            if what == "unembed":
                emb[n] = logits
            elif what == "embed":
                emb[n] = m.embed[torch.tensor(id_lists, dtype=torch.long, device=m.device)]
        return logits, {k: emb[k] for k in names}

    def __call__(self, input_ids, return_embeddings: bool = False, layer_names=None):
        return self.forward(input_ids, return_embeddings, layer_names)

    # ---- generation ------------------------------------------------------------
    def generate(self, prompt_seqs, n_tokens: int = 500, temperature: float = 1.0,
                 top_k: int = 4, top_p: float = 1.0, batched: bool = True,
                 cached_generation: bool = True, verbose: int = 1,
                 force_prompt_threshold: int | None = None, *,
                 seed: int | None = None) -> GenerationOutput:
        """Exactly `n_tokens` per prompt with vortex sampling semantics
        (evo2_flash/api.py:839-982): the prompts are prefilled in packed steps,
        then every step decodes one token per prompt from the paged mixer state
        and the attention cache.  `seed` seeds prompt i's sampler with seed + i.
        `cached_generation` and `force_prompt_threshold` are accepted and
        ignored (decoding always continues from the cached state)."""
        _sampling_args(temperature, top_k, top_p)
        if isinstance(prompt_seqs, str):
            prompt_seqs = [prompt_seqs]
        prompt_seqs = list(prompt_seqs)
        if n_tokens < 1:
            raise ValueError("n_tokens must be positive")
        ids = [self.tokenizer.tokenize(s) for s in prompt_seqs]
        for x in ids:
            if not x:
                raise ValueError("empty prompt")
            self._check_len(len(x) + n_tokens, "prompt + n_tokens")
        if not ids:
            return GenerationOutput(sequences=[], logprobs_mean=[])
        gens = [None if seed is None else torch.Generator().manual_seed(seed + i)
                for i in range(len(ids))]
        m = self.model
        last = [None] * len(ids)
        with torch.no_grad():
            for h, segs in m.prefill_steps([torch.tensor(x, dtype=torch.long) for x in ids],
                                           self.max_tokens_per_step, keep_cache=True):
                for a, b, sid, p0 in segs:
                    if p0 + (b - a) == len(ids[sid]):
                        last[sid] = h[b - 1]
            h = torch.stack(last)
            toks = [[] for _ in ids]
            lps = [[] for _ in ids]
            try:
                for step in range(n_tokens):
                    lg = F.linear(h, m.embed).float()
                    lp = torch.log_softmax(lg, -1)
                    nxt = [sample_token(lg[i], temperature, top_k, top_p, gens[i])
                           for i in range(len(ids))]
                    for i, t in enumerate(nxt):
                        toks[i].append(t)
                        lps[i].append(float(lp[i, t]))
                    if step + 1 < n_tokens:
                        h = m.decode_step(nxt, [len(x) + step for x in ids], range(len(ids)))
            finally:
                m.release_all()
        seqs = [self.tokenizer.detokenize(t) for t in toks]
        means = [sum(v) / len(v) for v in lps]
        uniform = all(len(x) == len(ids[0]) for x in ids)

        def logits_fn():
            per = []
            for p, t in zip(ids, toks):
                lg, _ = self.forward([p + t[:-1]])
                per.append(lg[0, len(p) - 1:].float())
            if batched and uniform:
                return [torch.stack(per)]
            return [x[None] for x in per]

        if verbose:
            for s, score, prompt in zip(seqs, means, prompt_seqs):
                print(f'Prompt: "{prompt}",\tOutput: "{s}",\tScore: {score}')
        return GenerationOutput(sequences=seqs, logprobs_mean=means, token_ids=toks,
                                _logits_fn=logits_fn)
