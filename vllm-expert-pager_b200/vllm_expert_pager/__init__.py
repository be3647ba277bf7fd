"""B200-native expert paging for vLLM MoE models (drop-in for vllm-expert-pager).

Modules: ``table`` / ``acquire`` (slot tables), ``gather`` (row copies and the
SSD request ring), ``codec`` (fp8-exponent Huffman records), ``store`` (RAM and
SSD tiers), ``pager`` (per-layer decode and working paths), ``experts`` /
``plugin`` (the vLLM hook), ``native`` (the C-ABI library).
"""
