def register() -> None:
    # Imported inside the function: experts.py needs a loaded vLLM (plugin.py of
    # the reference, kept as is: it is the vllm.general_plugins entry point).
    from vllm_expert_pager import experts

    experts.register()
