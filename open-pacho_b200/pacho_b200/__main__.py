from .command import main

raise SystemExit(main())
