"""GSQ: grid and schedules, GPTQ, Lion and the stage optimiser on the GPU."""
