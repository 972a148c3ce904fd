"""mxq.nn — putting Schemes into a model (placeholder until MXLinear / attend land)."""
