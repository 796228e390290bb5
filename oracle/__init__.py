"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the Whisper attention path (see oracle.py)."""
