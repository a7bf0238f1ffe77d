"""Per-``generate`` sampling configuration.

Field-for-field compatible with the reference ``SamplingParams``
(``nano_vllm_uno/sampling_params.py:4-64``) so that user code written for the
reference runs unchanged. Validation happens once in ``__post_init__``.
"""

from __future__ import annotations

from dataclasses import dataclass

NOISE_MODES = ("deterministic_uniform", "random_uniform", "mask")


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float | None = None
    top_k: int | None = None
    max_tokens: int = 64
    ignore_eos: bool = False
    stop_token_ids: list[int] | None = None
    # Diffusion-training mask token; draft noise is drawn from [1, mask_token_id).
    mask_token_id: int | None = None
    noise_mode: str = "random_uniform"
    noise_salt: int | None = None
    # Forward width including the seed token: 1 is plain autoregressive
    # decoding, L > 1 drafts L-1 tokens and verifies them (Psi-Spec).
    diffusion_block_size: int = 1
    # Base seed for the counter-based sampler RNG.  ``None`` draws one from the
    # engine's seed counter; a fixed value makes a run reproducible.
    seed: int | None = None

    def __post_init__(self) -> None:
        self.temperature = float(self.temperature)
        if self.temperature < 0.0:
            raise ValueError("temperature must be non-negative")
        if self.top_p is not None:
            self.top_p = float(self.top_p)
            if not 0.0 < self.top_p <= 1.0:
                raise ValueError("top_p must be in (0, 1] when provided")
        if self.top_k is not None:
            self.top_k = int(self.top_k)
            if self.top_p is not None and self.top_k <= 0:
                raise ValueError("top_k must be positive when provided with top_p")
        self.max_tokens = int(self.max_tokens)
        self.diffusion_block_size = int(self.diffusion_block_size)
        if self.diffusion_block_size < 1:
            raise ValueError("diffusion_block_size must be >= 1")
        if self.noise_mode not in NOISE_MODES:
            raise ValueError(
                f"Unsupported noise_mode={self.noise_mode!r}. "
                f"Expected one of {sorted(NOISE_MODES)}"
            )
        if self.mask_token_id is not None:
            self.mask_token_id = int(self.mask_token_id)
            if self.mask_token_id <= 1:
                raise ValueError("mask_token_id must be > 1 when provided")
        if (
            self.diffusion_block_size > 1
            and self.noise_mode == "mask"
            and self.mask_token_id is None
        ):
            raise ValueError(
                "Mask noise requires mask_token_id. Pass the diffusion-training "
                "mask token explicitly."
            )
        if self.stop_token_ids is not None:
            self.stop_token_ids = [int(t) for t in self.stop_token_ids]
        if self.noise_salt is not None:
            self.noise_salt = int(self.noise_salt)
        if self.seed is not None:
            self.seed = int(self.seed)

    # Derived properties used by the decoder dispatch.
    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0

    def uses_top_k(self, vocab_size: int) -> bool:
        return self.top_k is not None and 0 < int(self.top_k) < int(vocab_size)

    def uses_top_p(self) -> bool:
        return self.top_p is not None and 0.0 < float(self.top_p) < 1.0

    def filtered(self, vocab_size: int) -> bool:
        return self.uses_top_k(vocab_size) or self.uses_top_p()
