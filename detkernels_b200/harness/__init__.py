"""Pure result-aggregation helpers of the reference's harness (diff + sweep summaries).

Only the dependency-free parts are here: the vLLM audit (server, HTTP sweep,
activation localizer) is outside this library's scope."""
