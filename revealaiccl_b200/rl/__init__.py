"""Schedule-search RL stack: slot decoder, PPO, scenarios/evaluator, CLIs, XML export."""
