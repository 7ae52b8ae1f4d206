/*
 * gguf_synth_cli - the synthetic-model writer as a command:
 *
 *   pk_synth_cli OUT.gguf key=value ...
 *
 * with the keys of PksSpec (dim, hidden_dim, n_layers, n_heads, n_kv_heads,
 * vocab_size, context_length, rope_theta, rms_eps, weight_std, seed, t_embd,
 * t_output, t_q, t_k, t_v_even, t_v_odd, t_o, t_gate, t_up, t_down_even,
 * t_down_odd, tied_output, space_piece). Writes the same file as
 * pks_write_model (pk_synth.write_model) for the same spec, for callers that
 * prepare a model file without loading the writer into their own process.
 */
#include "gguf_synth.c"

int main(int argc, char **argv)
{
    if (argc < 2) {
        fprintf(stderr, "usage: %s OUT.gguf key=value ...\n", argv[0]);
        return 2;
    }
    PksSpec s;
    memset(&s, 0, sizeof(s));
    s.rms_eps = 1e-5f;
    s.weight_std = 0.02f;
    s.seed = 1234;
    for (int i = 2; i < argc; i++) {
        const char *eq = strchr(argv[i], '=');
        if (eq == NULL) {
            fprintf(stderr, "bad argument: %s\n", argv[i]);
            return 2;
        }
        const size_t kl = (size_t)(eq - argv[i]);
        const char *v = eq + 1;
#define INT_KEY(name)                                                     \
    if (kl == strlen(#name) && strncmp(argv[i], #name, kl) == 0) {        \
        s.name = (int)strtol(v, NULL, 10);                                \
        continue;                                                         \
    }
#define U32_KEY(name)                                                     \
    if (kl == strlen(#name) && strncmp(argv[i], #name, kl) == 0) {        \
        s.name = (uint32_t)strtoul(v, NULL, 10);                          \
        continue;                                                         \
    }
#define F32_KEY(name)                                                     \
    if (kl == strlen(#name) && strncmp(argv[i], #name, kl) == 0) {        \
        s.name = strtof(v, NULL);                                         \
        continue;                                                         \
    }
        INT_KEY(dim) INT_KEY(hidden_dim) INT_KEY(n_layers) INT_KEY(n_heads) INT_KEY(n_kv_heads)
        INT_KEY(vocab_size) INT_KEY(context_length) INT_KEY(tied_output) INT_KEY(space_piece)
        F32_KEY(rope_theta) F32_KEY(rms_eps) F32_KEY(weight_std)
        U32_KEY(t_embd) U32_KEY(t_output) U32_KEY(t_q) U32_KEY(t_k) U32_KEY(t_v_even) U32_KEY(t_v_odd)
        U32_KEY(t_o) U32_KEY(t_gate) U32_KEY(t_up) U32_KEY(t_down_even) U32_KEY(t_down_odd)
        if (kl == 4 && strncmp(argv[i], "seed", 4) == 0) {
            s.seed = (uint64_t)strtoull(v, NULL, 10);
            continue;
        }
        fprintf(stderr, "unknown key: %s\n", argv[i]);
        return 2;
    }
    char err[256] = {0};
    if (pks_write_model(argv[1], &s, err, sizeof(err)) != 1) {
        fprintf(stderr, "%s\n", err);
        return 1;
    }
    return 0;
}
