"""Drop-in build step -- TEST INFRASTRUCTURE ONLY.

Writes patched copies of the reference's src/inference/inference.h and
src/inference/inference.c into a build directory (oracle/_ref/dropin, never
committed) with the hook INTEGRATION.md describes, so that the reference's own
transformer_forward runs on libengine_cuda.so when a context is attached:

  inference.h: t_transformer gains `struct ec_ctx *gpu;` (last member, under
               ENGINE_CUDA; NULL keeps the CPU path);
  inference.c: `#include "../config.h"` becomes `#include "config.h"` (the
               copy lives outside src/), and transformer_forward starts with
               `if (t->gpu) return ec_forward(t, token, pos);`, where
               ec_forward calls ec_decode_step into t->state.logits.

Usage: python dropin.py <reference src dir> <out dir>
"""
import os
import sys

HOOK_FN = '''
#ifdef ENGINE_CUDA
# include "engine_cuda.h"
/* engine_cuda drop-in (INTEGRATION.md): the whole decode step on the GPU,
** logits copied into the reference's host buffer (inference.h:190). */
static float	*ec_forward(t_transformer *t, int token, int pos)
{
	int	rc;

	rc = ec_decode_step(t->gpu, &token, &pos, 1, t->state.logits, NULL);
	if (rc != EC_OK)
	{
		fprintf(stderr, "engine_cuda: %s\\n", ec_last_error());
		return (NULL);
	}
	return (t->state.logits);
}
#endif

'''

HOOK_CALL = '''#ifdef ENGINE_CUDA
	if (t->gpu)
		return (ec_forward(t, token, pos));
#endif
'''

SIGNATURE = "float\t*transformer_forward(t_transformer *t, int token, int pos)"


def patch(src_dir, out_dir):
    os.makedirs(os.path.join(out_dir, "inference"), exist_ok=True)
    h = open(os.path.join(src_dir, "inference", "inference.h")).read()
    end = h.index("}\tt_transformer;")
    h = h[:end] + "#ifdef ENGINE_CUDA\n\tstruct ec_ctx\t\t*gpu;\n#endif\n" + h[end:]
    c = open(os.path.join(src_dir, "inference", "inference.c")).read()
    if '#include "../config.h"' not in c or c.count(SIGNATURE) != 1:
        raise SystemExit("dropin: the reference's inference.c does not have the expected shape")
    c = c.replace('#include "../config.h"', '#include "config.h"', 1)
    at = c.index(SIGNATURE)
    brace = c.index("{", at) + 1
    c = c[:at] + HOOK_FN + c[at:brace] + "\n" + HOOK_CALL + c[brace:]
    for name, text in (("inference.h", h), ("inference.c", c)):
        with open(os.path.join(out_dir, "inference", name), "w") as f:
            f.write(text)


if __name__ == "__main__":
    patch(sys.argv[1], sys.argv[2])
