"""Shared XGrammar fixtures for the tests: a tokenizer of V tokens (printable ASCII characters, an
EOS token, then filler tokens "tok<N>") and a JSON-like grammar whose states range from a handful
of allowed tokens (punctuation, letters, digits) to nearly all of them (a free-text string)."""

PRINTABLE = [chr(c) for c in range(32, 127)]
EOS = len(PRINTABLE)
GRAMMAR = r'''root ::= "{" "\"" [a-z]+ "\"" ":" ( [0-9]+ | "\"" [^"]* "\"" ) "}"'''


def compiled(vocab: int):
    import xgrammar as xgr
    tokens = PRINTABLE + ["<eos>"] + [f"tok{i}" for i in range(vocab - len(PRINTABLE) - 1)]
    info = xgr.TokenizerInfo(tokens, stop_token_ids=[EOS])
    return xgr.GrammarCompiler(info, max_threads=4).compile_grammar(GRAMMAR)


def char(c: str) -> int:
    return ord(c) - 32
