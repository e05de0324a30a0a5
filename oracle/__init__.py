"""CPU oracle for the Gemma-4 MoE block (test infrastructure only)."""
