"""Engine: scheduler and the LLM engine loop."""
